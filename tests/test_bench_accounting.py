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
    import bench
    cfg = _cfg(pkg)
    ctx = bench.contexts(64, 0)
    out, _ = bench.stage_bytes(cfg, ctx, None)
    n_gdn = 36
    state = 32 * 128 * 128 * 4 * 2            # one sequence's state, read + written
    cd = 2 * 16 * 128 + 32 * 128
    history = 3 * cd * 4 * 2                   # conv history, read + written
    row = (cd + 32 * 128 + 2 * 32) * 4 + 32 * 128 * 2  # projection row in, bf16 output row
    assert out["RecurrentUpdate"] == n_gdn * 64 * (state + history + row)
    # the state dominates: 268.4 MB per layer for 64 sequences
    assert abs(64 * state / 1e6 - 268.4) < 0.1


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
