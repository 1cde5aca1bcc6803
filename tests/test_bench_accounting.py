"""bench.py's algorithmic byte accounting on CPU: the per-stage bytes that the
roofline fractions divide by. The DeltaNet term is the fp32 state read and
written once per (sequence, value head) plus the conv history and the token's
projection row; the MoE terms count each distinct expert's weights once per
layer; with expert parallelism the ranks' expert blocks partition the weights."""
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))


def _cfg(pkg):
    return pkg.config1()


def test_recurrent_update_bytes_cfg1(pkg):
    """The DeltaNet term equals what the library itself holds per sequence:
    the DeltaNet part of the reference-layout state (rs_qwen_state_count minus
    the attention K/V), read and written once per step, plus each token's
    projection row in and gated output row out."""
    import bench
    cfg = _cfg(pkg)
    ctx = bench.contexts(64, 0)
    out, _ = bench.stage_bytes(cfg, ctx, None)
    n_attn = cfg.layers // cfg.interval
    n_gdn = cfg.layers - n_attn
    kv_floats = n_attn * 2 * cfg.kv_heads * cfg.context * cfg.head_dim
    gdn_floats = pkg.state_count(cfg) - kv_floats  # conv history + recurrent state, all DeltaNet layers
    assert gdn_floats * 4 == bench.gdn_slot_bytes(cfg)  # the session's per-version DeltaNet slot
    in_row = (2 * cfg.key_heads * cfg.key_dim + 2 * cfg.value_heads * cfg.value_dim + 2 * cfg.value_heads) * 4
    out_row = cfg.value_heads * cfg.value_dim * 2
    assert out["RecurrentUpdate"] == n_gdn * 64 * (2 * gdn_floats * 4 // n_gdn + in_row + out_row)
    # the recurrent state dominates: 268.4 MB per layer for 64 sequences
    assert abs(64 * cfg.value_heads * cfg.value_dim * cfg.key_dim * 4 * 2 / 1e6 - 268.4) < 0.1


def test_chunk_tokens_add_rows_not_state(pkg):
    """Several tokens of one sequence in a step (prefill chunks, verify blocks)
    move the recurrent state once and one projection row per token; their K/V
    count once, at the final length."""
    import bench
    cfg = _cfg(pkg)
    ctx = np.array([100, 2000])
    one, _ = bench.stage_bytes(cfg, ctx, None)
    four, _ = bench.stage_bytes(cfg, ctx, None, counts=[4, 4])
    n_gdn = cfg.layers - cfg.layers // cfg.interval
    in_row = (2 * cfg.key_heads * cfg.key_dim + 2 * cfg.value_heads * cfg.value_dim + 2 * cfg.value_heads) * 4
    out_row = cfg.value_heads * cfg.value_dim * 2
    assert four["RecurrentUpdate"] - one["RecurrentUpdate"] == n_gdn * 6 * (in_row + out_row)
    kv = 2 * cfg.kv_heads * cfg.head_dim * 2 * (cfg.layers // cfg.interval)
    assert four["AttentionReduction"] - one["AttentionReduction"] == kv * 6 + (cfg.layers // cfg.interval) * 6 * (
        cfg.q_heads * 2 * cfg.head_dim + 2 * cfg.kv_heads * cfg.head_dim) * 4


def test_moe_bytes_count_distinct_experts(pkg):
    import bench
    cfg = _cfg(pkg)
    ctx = bench.contexts(64, 0)
    rng = np.random.default_rng(3)
    routing = rng.integers(0, cfg.experts, size=(cfg.layers, 64, cfg.top)).astype(np.int32)
    out, ue = bench.stage_bytes(cfg, ctx, routing)
    H, I, w = cfg.hidden, cfg.intermediate, bench.W4_BYTES_PER_PARAM
    distinct = np.array([len(np.unique(routing[l])) for l in range(cfg.layers)], np.float64) + 1
    rows = cfg.layers * 64 * (cfg.top + 1)
    assert np.isclose(out["MoeUpGate"], np.sum(distinct * 2 * I * H * w) + rows * (H * 2 + I * 2))
    assert np.isclose(out["MoeDown"], np.sum(distinct * H * I * w) + rows * (I * 2 + H * 4))
    assert np.isclose(ue, distinct.mean())


def test_expert_parallel_blocks_partition_the_weights(pkg):
    import bench
    cfg = _cfg(pkg)
    ctx = bench.contexts(64, 0)
    rng = np.random.default_rng(5)
    routing = rng.integers(0, cfg.experts, size=(cfg.layers, 128, cfg.top)).astype(np.int32)
    H, I, w = cfg.hidden, cfg.intermediate, bench.W4_BYTES_PER_PARAM
    whole = sum(len(np.unique(routing[l])) for l in range(cfg.layers))
    per = cfg.experts // 2
    parts = 0.0
    for rank in range(2):
        out, ue = bench.stage_bytes(cfg, ctx, routing, (rank * per, (rank + 1) * per))
        parts += (ue - 1) * cfg.layers
    # every distinct routed expert is counted by exactly one rank
    assert np.isclose(parts, whole)


def test_per_launch_bytes_follow_the_layer_count(pkg):
    """The roofline's bytes per launch divide a stage's step bytes by the
    launches of its kernel in that step: one per layer of the stage's kind, so
    a 4-layer slice reports the same per-launch bytes as the 48-layer model."""
    import bench
    ctx = bench.contexts(64, 0)
    per = {}
    for layers in (48, 4):
        cfg = pkg.config1(layers=layers)
        out, _ = bench.stage_bytes(cfg, ctx, None)
        per[layers] = {k: out[k] / bench.launches_per_step(k, cfg)
                       for k in ("MoeUpGate", "MoeDown", "RecurrentUpdate", "AttentionReduction")}
    for k in per[48]:
        assert np.isclose(per[48][k], per[4][k]), k
