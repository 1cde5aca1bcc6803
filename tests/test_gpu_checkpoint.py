"""Models built from MLX-layout safetensors checkpoints (rs_mlx_weights_load +
rs_qwen_quant) on the device, at configs[0] widths:
  - a 4-bit g64 checkpoint holding the synthetic weights gives, bit for bit,
    the logits of the synthetic store (the loader writes the same tiles);
  - a checkpoint with 8-bit routers and shared-expert gates (the Combined
    model's override, native/qwen_model.inc:273-276), RMSNorm gains stored as
    offsets from 1 and conv weights in [channels, 1, taps] layout matches the
    FP64 oracle given the same 8-bit rows (rel-L2 <= 1e-2), and its tensors
    still export byte for byte after the device layout is built."""
import numpy as np
import pytest

from checkpoint_util import checkpoint_tensors, quantize_rows, write_safetensors
from conftest import has_cuda

pytestmark = pytest.mark.gpu


def rel_l2(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def prefill_decode(pkg, sess, cfg, seed=3):
    rng = np.random.default_rng(seed)
    lens = [7, 19, 40]
    toks = [rng.integers(0, cfg.vocab, size=n).astype(np.uint32) for n in lens]
    sess.set_capture(True)
    outs, first, _ = sess.step_ragged([None] * 3, [0] * 3, lens, np.concatenate(toks))
    route_p = sess.debug_routing(sum(lens))
    outs2, tok2, logits = sess.step_ragged(outs, lens, [1] * 3, first, flags=pkg.RAGGED_SAMPLED | pkg.RAGGED_LOGITS)
    route_d = sess.debug_routing(3)
    for o in outs + outs2:
        sess.release(o)
    return lens, toks, first, logits, route_p, route_d


def test_checkpoint_equals_synthetic_store(pkg, O, tmp_path):
    if not has_cuda():
        pytest.skip("no CUDA device")
    cfg = pkg.config0()
    model = O.Model(O.config0(), 9)
    write_safetensors(tmp_path / "m.safetensors", checkpoint_tensors(O.config0(), model))
    loaded = pkg.WeightStore().load(tmp_path / "m.safetensors")
    synth = pkg.WeightStore().synthetic(cfg, 9)
    s1 = pkg.DeviceSession(loaded, cfg, slots=16, budget_bytes=1 << 30)
    s2 = pkg.DeviceSession(synth, cfg, slots=16, budget_bytes=1 << 30)
    try:
        r1 = prefill_decode(pkg, s1, cfg)
        r2 = prefill_decode(pkg, s2, cfg)
        assert np.array_equal(r1[3], r2[3])
        assert np.array_equal(r1[2], r2[2])
    finally:
        s1.close()
        s2.close()
        loaded.close()
        synth.close()


def test_checkpoint_with_8bit_routers_matches_oracle(pkg, O, tmp_path):
    if not has_cuda():
        pytest.skip("no CUDA device")
    O.set_routing_slack(5e-2)
    cfg, ocfg = pkg.config0(), O.config0()
    model = O.Model(ocfg, 10)
    rng = np.random.default_rng(6)
    ov = {}
    for i in range(cfg.layers):
        for name, rows in ((f"language_model.model.layers.{i}.mlp.gate", cfg.experts),
                           (f"language_model.model.layers.{i}.mlp.shared_expert_gate", 1)):
            ov[name] = quantize_rows(rng, rows, cfg.hidden, 8, 64) + (8,)
            model.override(name, 8, 64, *ov[name][:3])
    tensors = checkpoint_tensors(ocfg, model, overrides=ov, shifted=True)
    write_safetensors(tmp_path / "m.safetensors", tensors)
    store = pkg.WeightStore().load(tmp_path / "m.safetensors")
    for name in ov:
        store.quant(name, 64, 8)
    sess = pkg.DeviceSession(store, cfg, slots=16, budget_bytes=1 << 30)
    try:
        lens, toks, first, logits, route_p, route_d = prefill_decode(pkg, sess, cfg)
        cu = np.concatenate([[0], np.cumsum(lens)])
        for s in range(3):
            _, st, _, _ = model.forward(toks[s], 0, forced_routing=route_p[:, cu[s]:cu[s + 1]])
            lg, _, _, _ = model.forward([first[s]], lens[s], old_state=st, forced_routing=route_d[:, s:s + 1])
            assert rel_l2(logits[s], lg[0]) <= 1e-2, (s, rel_l2(logits[s], lg[0]))
        for name, arr, dt in tensors[:40]:
            raw = np.ascontiguousarray(arr).tobytes()
            assert store.weight_bytes(name, 0, len(raw), {"F32": 0, "U32": 2, "BF16": 4}[dt]) == raw, name
    finally:
        sess.close()
        store.close()
