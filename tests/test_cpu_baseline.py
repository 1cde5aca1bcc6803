"""The timed CPU baseline (oracle/fp32_step.cpp) computes the same decode step
as the FP64 oracle: configs[0], 8 sequences prefilled by the oracle, one
batched fp32 decode token per sequence, logits within rel-L2 1e-3 and the same
greedy tokens. CPU only."""
import numpy as np


def rel_l2(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def test_fp32_batched_step_matches_fp64_oracle(O):
    cfg = O.config0()
    model = O.Model(cfg, 21)
    rng = np.random.default_rng(8)
    lens = rng.integers(1, 257, size=8)
    states, toks = [], []
    for L in lens:
        prompt = rng.integers(0, cfg.vocab, size=int(L)).astype(np.uint32)
        _, st, _, _ = model.forward(prompt, 0)
        states.append(st)
        toks.append(int(rng.integers(0, cfg.vocab)))
    step = O.F32Step(cfg, 21, threads=4)
    step.set_batch(lens, np.stack(states), extra=4)
    sampled, logits, t_layers, t_head = step.step(toks, want_logits=True)
    assert t_layers > 0 and t_head > 0
    for s in range(8):
        lg, _, _, _ = model.forward([toks[s]], int(lens[s]), old_state=states[s])
        assert rel_l2(logits[s], lg[0]) <= 1e-3, (s, rel_l2(logits[s], lg[0]))
        assert int(sampled[s]) == int(np.argmax(lg[0]))
