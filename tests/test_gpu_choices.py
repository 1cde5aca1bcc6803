"""Constrained greedy selection on the device (rs_qwen_device_step_ragged_choices)
against the oracle's restatement of src/serving/choices.rs:65-98 applied to the
device's own logits: the legal id with the largest logit, lowest id on ties,
ids in any order and repeated; rows without a set fall back to the plain
greedy token; the step's states equal an unconstrained step's (selection is
output-only)."""
import numpy as np
import pytest

from conftest import has_cuda

pytestmark = pytest.mark.gpu


def test_choices_match_oracle_select(pkg, O):
    if not has_cuda():
        pytest.skip("no CUDA device")
    cfg = pkg.config0()
    store = pkg.WeightStore().synthetic(cfg, 31)
    sess = pkg.DeviceSession(store, cfg, slots=32, budget_bytes=1 << 30)
    try:
        rng = np.random.default_rng(4)
        lens = [3, 9, 17, 1, 30]
        toks = np.concatenate([rng.integers(0, cfg.vocab, size=n) for n in lens]).astype(np.uint32)
        flags = pkg.RAGGED_SAMPLED | pkg.RAGGED_LOGITS | pkg.RAGGED_ALL_ROWS
        rows = sum(lens)
        allowed = []
        for r in range(rows):
            k = r % 5
            if k == 0:
                allowed.append(None)  # unconstrained row
            elif k == 1:
                allowed.append([int(rng.integers(0, cfg.vocab))])
            elif k == 2:
                ids = rng.choice(cfg.vocab, size=40, replace=False)
                allowed.append(list(ids[::-1]) + list(ids[:5]))  # reversed, with repeats
            else:
                allowed.append(list(rng.integers(0, cfg.vocab, size=int(rng.integers(2, 300)))))
        outs, sampled, logits = sess.step_ragged_choices([None] * 5, [0] * 5, lens, toks, allowed, flags=flags)
        ref_outs, ref_sampled, ref_logits = sess.step_ragged([None] * 5, [0] * 5, lens, toks, flags=flags)
        assert np.array_equal(logits, ref_logits)
        for r in range(rows):
            want = int(ref_sampled[r]) if allowed[r] is None else O.select(logits[r], allowed[r])
            assert int(sampled[r]) == want, (r, allowed[r])
        for a, b in zip(outs, ref_outs):
            assert np.array_equal(sess.snapshot(a), sess.snapshot(b))
        for o in outs + ref_outs:
            sess.release(o)
        with pytest.raises(pkg.NativeError, match="invalid legal token"):
            sess.step_ragged_choices([None], [0], [2], toks[:2], [[cfg.vocab]])
        assert sess.stats()[0] == 0  # the rejected step reserved nothing
    finally:
        sess.close()
        store.close()
