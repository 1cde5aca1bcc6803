"""rs_qwen_forward (the reference's one-shot forward, native/qwen_model.inc:278-377)
through the C ABI at configs[0] widths.

It runs the session's ragged step on a private session after importing the
caller's reference-layout state, so a prompt fed in chunks of <= 8 tokens must
give, bit for bit, the logits and states of the same chunks stepped through a
device session (the import / export round trip is exact: K/V come back from
the bf16 cache they were read from, DeltaNet state is fp32 both ways). The
chain is also compared with the FP64 oracle fed the device's routing (rel-L2
<= 1e-2 for logits and state).
"""
import numpy as np
import pytest

from conftest import has_cuda

pytestmark = pytest.mark.gpu


def rel_l2(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def test_forward_chunks_match_session_and_oracle(pkg, O):
    if not has_cuda():
        pytest.skip("no CUDA device")
    O.set_routing_slack(5e-2)
    cfg = pkg.config0()
    store = pkg.WeightStore().synthetic(cfg, 77)
    sess = pkg.DeviceSession(store, cfg, slots=16, budget_bytes=1 << 30)
    model = O.Model(O.config0(), 77)
    try:
        toks = np.random.default_rng(5).integers(0, cfg.vocab, size=21).astype(np.uint32)
        chunks = [toks[:8], toks[8:16], toks[16:20], toks[20:]]
        state_f, state_o, parent, off = None, None, None, 0
        sess.set_capture(True)
        for ch in chunks:
            logits_f, new_f = store.forward(cfg, ch, off, old_state=state_f)
            (child,), _, logits_s = sess.step_ragged([parent], [off], [len(ch)], ch, flags=pkg.RAGGED_LOGITS)
            route = sess.debug_routing(len(ch))
            snap = sess.snapshot(child)
            assert np.array_equal(logits_f, logits_s[0])
            assert np.array_equal(new_f, snap)
            lg, state_o, _, _ = model.forward(ch, off, old_state=state_o, forced_routing=route)
            assert rel_l2(logits_f, lg[-1]) <= 1e-2
            assert rel_l2(new_f, state_o) <= 1e-2
            if parent is not None:
                sess.release(parent)
            parent, state_f, off = child, new_f, off + len(ch)
        sess.release(parent)
        # argument checks of the reference contract
        with pytest.raises(pkg.NativeError, match="state length"):
            store.forward(cfg, toks[:2], 3, old_state=np.zeros(5, np.float32))
        with pytest.raises(pkg.NativeError, match="geometry"):
            store.forward(cfg, toks[:9], 0)  # more than chunk (8) tokens
    finally:
        sess.close()
        store.close()
