"""tcgen05 4-bit GEMM engine vs the CUDA-core engine on identical inputs.

The CUDA-core engine dequantises in fp32 and is pinned to the FP64 oracle by
the model-level parity tests; the tcgen05 engine rounds each dequantised
weight once to IEEE half (the MMA operand type, 11 significant bits), so the
two agree to half precision: rel-L2 <= 1e-3 per launch.
"""
import numpy as np
import pytest

from conftest import has_cuda

pytestmark = pytest.mark.gpu


def f16_bits(a):
    return np.asarray(a, np.float32).astype(np.float16).view(np.uint16)


def rel(a, b):
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.mark.parametrize("widths", ["cfg0", "cfg1"])
def test_tc_engine_matches_cuda_core_engine(pkg, widths):
    if not has_cuda():
        pytest.skip("no CUDA device")
    if widths == "cfg0":
        cfg = pkg.config0()
        layers = [0, 3]
    else:
        cfg = pkg.config1(layers=4, context=1024)
        layers = [0, 3]
    store = pkg.WeightStore().synthetic(cfg, 99)
    sess = pkg.DeviceSession(store, cfg, slots=8, budget_bytes=4 << 30)
    rng = np.random.default_rng(3)
    H = cfg.hidden
    vd = cfg.value_heads * cfg.value_dim
    hq = cfg.q_heads * cfg.head_dim
    try:
        for layer in layers:
            attn = (layer + 1) % cfg.interval == 0
            in_rows = (cfg.q_heads * 2 * cfg.head_dim + 2 * cfg.kv_heads * cfg.head_dim) if attn else \
                (2 * cfg.key_heads * cfg.key_dim + 2 * vd + 2 * cfg.value_heads)
            for which, k, rows in ((0, H, in_rows), (1, hq if attn else vd, H), (2, H, cfg.experts + 1),
                                   (3, H, cfg.vocab)):
                if which == 3 and layer != layers[0]:
                    continue
                for T in (1, 5, 16, 30, 64, 130):
                    if which == 3 and T > 64:
                        continue
                    x = f16_bits(rng.standard_normal((T, k)))
                    y_tc, ms_tc = sess.debug_gemm(which, layer, x, rows, engine=0)
                    y_ref, _ = sess.debug_gemm(which, layer, x, rows, engine=1)
                    err = rel(y_tc, y_ref)
                    assert err < 1e-3, (widths, layer, which, T, err)
    finally:
        sess.close()
        store.close()
