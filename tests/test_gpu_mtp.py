"""MTP draft head (rs_qwen_device_mtp_attach / _step / _snapshot / _release)
against the oracle's MTP forward (native/qwen_mtp.inc:29-46 semantics:
fc(concat(rms(embed(tok)), rms(target hidden))) -> attention layer with its own
KV -> MoE -> norm -> target lm_head).

The device's MTP routing is fed to the oracle (checked there to be a top-k of
the FP64 logits within the slack), so the comparison isolates the arithmetic:
last-row logits, the draft's hidden rows and its KV within rel-L2 1e-2, greedy
token equal. The autoregressive step (draft_source = 1) is checked from the
device's own draft state (KV and last hidden row), so each step's error is
measured on its own. Runs at configs[0] and at configs[1] widths.
"""
import numpy as np
import pytest

from conftest import has_cuda

pytestmark = pytest.mark.gpu

TOL = 1e-2
ROUTING_SLACK = 5e-2


def rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.fixture(scope="module", params=["cfg0", "cfg1"])
def mtp(pkg, O, request):
    """configs[0], and configs[1] widths (hidden 2048, 512 experts top-10,
    16q/2kv/256, vocab 151936) on a 4-layer slice plus the MTP layer."""
    if not has_cuda():
        pytest.skip("no CUDA device")
    if request.param == "cfg0":
        cfg, ocfg = pkg.config0(), O.config0()
    else:
        cfg, ocfg = pkg.config1(layers=4, context=1024), O.config1(layers=4, context=1024)
    store = pkg.WeightStore().synthetic(cfg, 21, mtp=True)
    sess = pkg.DeviceSession(store, cfg, slots=32, budget_bytes=4 << 30)
    sess.mtp_attach(store)
    model = O.Model(ocfg, 21, mtp=True)
    O.set_routing_slack(ROUTING_SLACK)
    yield pkg, cfg, sess, model
    sess.close()
    store.close()


def test_mtp_steps_match_oracle(mtp, O):
    pkg, cfg, sess, model = mtp
    rng = np.random.default_rng(5)
    n = 6
    prompt = rng.integers(0, cfg.vocab, size=n).astype(np.uint32)
    outs, _, _ = sess.step_ragged([None], [0], [n], prompt, flags=pkg.RAGGED_SAMPLED | pkg.RAGGED_HIDDEN)
    target = outs[0]
    hidden = sess.hidden_snapshot(target, n)
    toks = rng.integers(0, cfg.vocab, size=n).astype(np.uint32)

    sess.set_capture(True)
    d1, lg1 = sess.mtp_step(None, target, toks, row=0)
    routing = sess.debug_routing(n)[0]
    sess.set_capture(False)
    kv = np.zeros(2 * cfg.kv_heads * cfg.context * cfg.head_dim, np.float64)
    lo, ho = model.mtp_forward(toks, 0, hidden.astype(np.float64), kv, forced_routing=routing)
    assert d1.position == n
    assert rel(lg1, lo[-1]) <= TOL
    assert int(np.argmax(lg1)) == int(np.argmax(lo[-1]))
    k1, v1, h1 = sess.mtp_snapshot(d1, n)
    kvo = kv.reshape(2, cfg.kv_heads, cfg.context, cfg.head_dim)
    assert rel(h1, ho) <= TOL
    assert rel(k1[:, :n], kvo[0][:, :n]) <= TOL and rel(v1[:, :n], kvo[1][:, :n]) <= TOL
    assert not np.any(k1[:, n:]) and not np.any(v1[:, n:])

    # autoregressive draft token from the draft's own last hidden row
    t = int(np.argmax(lg1))
    sess.set_capture(True)
    d2, lg2 = sess.mtp_step(d1, d1, [t], row=n - 1, draft_source=1)
    routing2 = sess.debug_routing(1)[0]
    sess.set_capture(False)
    kv_dev = np.stack([k1, v1]).astype(np.float64).ravel().copy()
    lo2, ho2 = model.mtp_forward([t], n, h1[n - 1:n].astype(np.float64), kv_dev, forced_routing=routing2)
    assert d2.position == n + 1
    assert rel(lg2, lo2[0]) <= TOL
    k2, v2, h2 = sess.mtp_snapshot(d2, 1)
    assert rel(h2, ho2) <= TOL
    # the draft pool shares d1's pages: its first n positions are unchanged
    assert np.array_equal(k2[:, :n], k1[:, :n]) and np.array_equal(v2[:, :n], v1[:, :n])
    sess.mtp_release(d2)
    sess.mtp_release(d1)
    sess.release(target)


def test_mtp_rejects_bad_sources(mtp):
    pkg, cfg, sess, model = mtp
    rng = np.random.default_rng(6)
    prompt = rng.integers(0, cfg.vocab, size=4).astype(np.uint32)
    outs, _, _ = sess.step_ragged([None], [0], [4], prompt, flags=pkg.RAGGED_SAMPLED | pkg.RAGGED_HIDDEN)
    with pytest.raises(pkg.NativeError, match="alignment"):
        sess.mtp_step(None, outs[0], prompt[:2], row=1)  # hidden row 1 is position 1, not 0
    d1, _ = sess.mtp_step(None, outs[0], prompt, row=0)
    with pytest.raises(pkg.NativeError, match="autoregressive"):
        sess.mtp_step(d1, d1, prompt[:2], row=3, draft_source=1)  # autoregressive steps take one token
    sess.mtp_release(d1)
    sess.release(outs[0])
