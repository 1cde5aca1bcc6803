"""rs_qwen_project_noalloc (allocation-free dense projection, split partials in
a static device array) against rs_qwen_debug_gemm (the session-buffer path)
on the same inputs, through the C ABI.

Both run the tcgen05 split-K GEMM with the same split choice and sum the
partials in the same order, so they agree to rounding (asserted: rel-L2 and
max-abs within 1e-6 relative); two calls in a row check that one call's
leftovers in the shared scratch do not reach the next. Collected last so it
also runs after every other GPU test in one process.
"""
import numpy as np
import pytest

from conftest import has_cuda

pytestmark = pytest.mark.gpu

TOL = 1e-6


def f16_bits(a):
    """IEEE-half bits: the projection input type."""
    return np.asarray(a, np.float32).astype(np.float16).view(np.uint16)


def rel(a, b):
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def noalloc(sess, which, layer, x_bits, rows):
    import torch
    T = x_bits.shape[0]
    xd = torch.from_numpy(x_bits.view(np.int16)).cuda()
    yd = torch.full((T, rows), float("nan"), dtype=torch.float32, device="cuda")
    torch.cuda.synchronize()
    sess.project_noalloc(which, layer, xd.data_ptr(), T, yd.data_ptr(), T * rows)
    return yd.cpu().numpy()


def in_rows(cfg, layer):
    attn = (layer + 1) % cfg.interval == 0
    if attn:
        return cfg.q_heads * 2 * cfg.head_dim + 2 * cfg.kv_heads * cfg.head_dim, cfg.q_heads * cfg.head_dim
    vd = cfg.value_heads * cfg.value_dim
    return 2 * cfg.key_heads * cfg.key_dim + 2 * vd + 2 * cfg.value_heads, vd


@pytest.mark.parametrize("widths", ["cfg0", "cfg1"])
def test_noalloc_projection_matches_session_path(pkg, widths):
    if not has_cuda():
        pytest.skip("no CUDA device")
    cfg = pkg.config0() if widths == "cfg0" else pkg.config1(layers=4, context=1024)
    store = pkg.WeightStore().synthetic(cfg, 99)
    sess = pkg.DeviceSession(store, cfg, slots=8, budget_bytes=4 << 30)
    rng = np.random.default_rng(17)
    H = cfg.hidden
    try:
        for layer in (0, 3):
            rows_in, k_out = in_rows(cfg, layer)
            for which, k, rows in ((0, H, rows_in), (1, k_out, H), (2, H, cfg.experts + 1), (3, H, cfg.vocab)):
                for T in (1, 5, 64):
                    if T * rows > 4194240:  # beyond the static scratch (checked in the test below)
                        continue
                    # two calls in a row on different inputs, each against the session path
                    for _ in range(2):
                        x = f16_bits(rng.standard_normal((T, k)))
                        y_ref, _ = sess.debug_gemm(which, layer, x, rows, engine=0)
                        y = noalloc(sess, which, layer, x, rows)
                        assert np.all(np.isfinite(y)), (widths, layer, which, T)
                        assert rel(y, y_ref) <= TOL, (widths, layer, which, T, rel(y, y_ref))
                        assert np.max(np.abs(y - y_ref)) <= TOL * max(1.0, float(np.max(np.abs(y_ref))))
    finally:
        sess.close()
        store.close()


def test_noalloc_rejects_calls_beyond_the_scratch(pkg):
    if not has_cuda():
        pytest.skip("no CUDA device")
    import torch
    cfg = pkg.config0()
    store = pkg.WeightStore().synthetic(cfg, 5)
    sess = pkg.DeviceSession(store, cfg, slots=4, budget_bytes=1 << 30)
    try:
        T = 4194240 // cfg.vocab + 1  # lm_head: T x vocab floats one row past the 16 MiB scratch
        xd = torch.zeros((T, cfg.hidden), dtype=torch.int16, device="cuda")
        yd = torch.zeros((T, cfg.vocab), dtype=torch.float32, device="cuda")
        torch.cuda.synchronize()
        with pytest.raises(pkg.NativeError, match="scratch"):
            sess.project_noalloc(3, 0, xd.data_ptr(), T, yd.data_ptr(), T * cfg.vocab)
        # the entry point stays usable after a rejection
        x = f16_bits(np.random.default_rng(1).standard_normal((3, cfg.hidden)))
        y_ref, _ = sess.debug_gemm(3, 0, x, cfg.vocab, engine=0)
        assert rel(noalloc(sess, 3, 0, x, cfg.vocab), y_ref) <= TOL
    finally:
        sess.close()
        store.close()


def test_noalloc_on_a_second_device_keeps_the_callers_device(pkg):
    """A session on device 1 driven from a thread whose current device is 0:
    the entry point sets up device 1's kernels and scratch, matches the
    session path there, and leaves the caller on device 0."""
    if not has_cuda():
        pytest.skip("no CUDA device")
    import torch
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    cfg = pkg.config0()
    torch.cuda.set_device(1)
    store = pkg.WeightStore().synthetic(cfg, 5)
    sess = pkg.DeviceSession(store, cfg, slots=4, budget_bytes=1 << 30)
    try:
        x = f16_bits(np.random.default_rng(2).standard_normal((5, cfg.hidden)))
        y_ref, _ = sess.debug_gemm(0, 0, x, in_rows(cfg, 0)[0], engine=0)
        xd = torch.from_numpy(x.view(np.int16)).to("cuda:1")
        rows = in_rows(cfg, 0)[0]
        yd = torch.full((5, rows), float("nan"), dtype=torch.float32, device="cuda:1")
        torch.cuda.synchronize(1)
        torch.cuda.set_device(0)
        for _ in range(2):
            sess.project_noalloc(0, 0, xd.data_ptr(), 5, yd.data_ptr(), 5 * rows)
            assert torch.cuda.current_device() == 0
            assert rel(yd.cpu().numpy(), y_ref) <= TOL
    finally:
        sess.close()
        store.close()
        torch.cuda.set_device(0)
