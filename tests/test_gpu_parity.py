"""GPU parity: the CUDA path through the C ABI against the CPU oracle.

Tolerances (north star): logits rel-L2 <= 1e-2 per row, greedy argmax agreement
>= 99% where the oracle's top-2 margin exceeds the numerical noise floor;
integer outputs (weight bytes, routing given identical logits) bit-exact.
The oracle is fed the device's expert selection (captured per step), as the
reference's own routing probe validates MLX's selection rather than
recomputing it (native/operator_probe.inc:19-23); the oracle checks that the
selection is a top-k of its FP64 router logits.
"""
import numpy as np
import pytest

from conftest import has_cuda

pytestmark = pytest.mark.gpu

SEED = 1234


def rel_l2(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


@pytest.fixture(scope="module")
def cuda_ok():
    if not has_cuda():
        pytest.skip("no CUDA device")


# The oracle checks the device's forced expert selection against its own FP64
# router logits. 16-bit GEMM operands (fp16 dequantised weights and
# activations) move router logits by ~1e-3 after a few layers, and experts tie
# within that.
ROUTING_SLACK = 5e-2


@pytest.fixture(autouse=True)
def _fresh_session_state(request):
    """Each test starts from an empty state table (a failed test leaks no versions)."""
    for name in ("tiny", "wide"):
        if name in request.fixturenames:
            request.getfixturevalue(name)[3].drain()
    yield


@pytest.fixture(scope="module")
def tiny(pkg, O, cuda_ok):
    O.set_routing_slack(ROUTING_SLACK)
    cfg = pkg.config0()
    store = pkg.WeightStore().synthetic(cfg, SEED)
    sess = pkg.DeviceSession(store, cfg, slots=64, budget_bytes=4 << 30)
    model = O.Model(O.config0(), SEED)
    yield pkg, cfg, store, sess, model
    sess.close()
    store.close()


def test_weight_bytes_bit_exact(tiny):
    pkg, cfg, store, sess, model = tiny
    names = [("language_model.model.embed_tokens", cfg.vocab, cfg.hidden),
             ("language_model.lm_head", cfg.vocab, cfg.hidden),
             ("language_model.model.layers.0.linear_attn.in_proj_qkv", 2 * 2 * 64 + 4 * 64, cfg.hidden),
             ("language_model.model.layers.0.linear_attn.in_proj_b", 4, cfg.hidden),
             ("language_model.model.layers.3.self_attn.q_proj", 4 * 2 * 64, cfg.hidden),
             ("language_model.model.layers.3.self_attn.v_proj", 64, cfg.hidden),
             ("language_model.model.layers.2.mlp.switch_mlp.gate_proj", 16 * 128, cfg.hidden),
             ("language_model.model.layers.2.mlp.switch_mlp.up_proj", 16 * 128, cfg.hidden),
             ("language_model.model.layers.2.mlp.switch_mlp.down_proj", 16 * cfg.hidden, 128),
             ("language_model.model.layers.1.mlp.shared_expert_gate", 1, cfg.hidden),
             ("language_model.model.layers.1.mlp.shared_expert.up_proj", 128, cfg.hidden)]
    for name, rows, cols in names:
        n = min(rows, 300)
        r0 = rows - n
        packed, sc, bi = model.qrows(name, r0, n, cols)
        dev_w = np.frombuffer(store.weight_bytes(name + ".weight", r0 * cols // 2, n * cols // 2), np.uint32)
        dev_s = np.frombuffer(store.weight_bytes(name + ".scales", r0 * cols // 16, n * cols // 16, 0), np.float32)
        dev_b = np.frombuffer(store.weight_bytes(name + ".biases", r0 * cols // 16, n * cols // 16, 0), np.float32)
        assert np.array_equal(dev_w, packed.ravel()), name
        assert np.array_equal(dev_s, sc.ravel()), name
        assert np.array_equal(dev_b, bi.ravel()), name
    for vname, n in (("language_model.model.layers.0.linear_attn.A_log", 4),
                     ("language_model.model.layers.2.linear_attn.conv1d.weight", 512 * 4)):
        dev = np.frombuffer(store.weight_bytes(vname, 0, 4 * n, 0), np.float32)
        assert np.array_equal(dev, model.vector(vname, n)), vname


def _prefix_batch(seed, n, vocab, lo=1, hi=256):
    rng = np.random.default_rng(seed)
    lens = rng.integers(lo, hi + 1, size=n)
    toks = [rng.integers(0, vocab, size=int(L)).astype(np.uint32) for L in lens]
    return lens, toks


def test_cfg0_prefill_then_decode_matches_oracle(tiny):
    """8 sequences, prefixes U[1, 256], one greedy decode token."""
    _prefill_then_decode(*tiny)


def test_conv3_prefill_then_decode_matches_oracle(pkg, O, cuda_ok):
    """configs[0] with a 3-tap DeltaNet conv (the conv width is a runtime
    parameter of the DeltaNet kernels; every preset uses 4)."""
    O.set_routing_slack(ROUTING_SLACK)
    cfg, ocfg = pkg.config0(), O.config0()
    cfg.conv = ocfg.conv = 3
    store = pkg.WeightStore().synthetic(cfg, SEED)
    sess = pkg.DeviceSession(store, cfg, slots=64, budget_bytes=4 << 30)
    try:
        _prefill_then_decode(pkg, cfg, store, sess, O.Model(ocfg, SEED))
    finally:
        sess.close()
        store.close()


def _prefill_then_decode(pkg, cfg, store, sess, model):
    lens, toks = _prefix_batch(0, 8, cfg.vocab)
    sess.set_capture(True)
    outs, sampled, _ = sess.step_ragged([None] * 8, [0] * 8, lens, np.concatenate(toks),
                                        flags=pkg.RAGGED_SAMPLED)
    T = int(lens.sum())
    route_prefill = sess.debug_routing(T)
    cu = np.concatenate([[0], np.cumsum(lens)])
    # oracle prefill with the device's expert selection
    o_states, o_first = [], []
    for s in range(8):
        lg, st, _, _ = model.forward(toks[s], 0, forced_routing=route_prefill[:, cu[s]:cu[s + 1], :])
        o_states.append(st)
        o_first.append(int(np.argmax(lg[-1])))
    # state after prefill: snapshot vs oracle state
    for s in range(8):
        snap = sess.snapshot(outs[s])
        assert rel_l2(snap, o_states[s]) < 1e-2, (s, rel_l2(snap, o_states[s]))
    # one decode token (the device's greedy token) for every sequence
    nxt = sampled.astype(np.uint32)
    outs2, sampled2, logits = sess.step_ragged(outs, lens, [1] * 8, nxt,
                                               flags=pkg.RAGGED_SAMPLED | pkg.RAGGED_LOGITS)
    route_dec = sess.debug_routing(8)
    for s in range(8):
        lg, _, _, _ = model.forward([nxt[s]], int(lens[s]), old_state=o_states[s],
                                    forced_routing=route_dec[:, s:s + 1, :])
        err = rel_l2(logits[s], lg[0])
        assert err < 1e-2, (s, err)
        assert sampled2[s] == int(np.argmax(logits[s]))
    # the greedy-agreement gate (>= 99 % of tokens) is asserted over 192 tokens
    # in test_gpu_bench_parity.py
    for o in list(outs) + list(outs2):
        sess.release(o)
    assert sess.stats()[0] == 0


def test_cfg0_ragged_mixed_step_equals_separate_steps(tiny):
    """A mixed prefill+decode ragged step gives the same tokens and states as
    running each sequence alone (batch composition must not change results)."""
    pkg, cfg, store, sess, model = tiny
    lens, toks = _prefix_batch(5, 6, cfg.vocab, 1, 40)
    outs, sampled, logits = sess.step_ragged([None] * 6, [0] * 6, lens, np.concatenate(toks),
                                             flags=pkg.RAGGED_SAMPLED | pkg.RAGGED_LOGITS)
    for s in range(6):
        o1, s1, l1 = sess.step_ragged([None], [0], [lens[s]], toks[s], flags=pkg.RAGGED_SAMPLED | pkg.RAGGED_LOGITS)
        assert s1[0] == sampled[s]
        assert np.array_equal(l1[0], logits[s])
        assert np.array_equal(sess.snapshot(o1[0]), sess.snapshot(outs[s]))
        sess.release(o1[0])
    for o in outs:
        sess.release(o)


def test_cfg0_branching_and_release(tiny):
    """Two children of one parent (copy-on-write of the shared partial page)
    are independent; releasing the parent keeps the children valid."""
    pkg, cfg, store, sess, model = tiny
    rng = np.random.default_rng(9)
    prefix = rng.integers(0, cfg.vocab, size=21).astype(np.uint32)
    (p,), _, _ = sess.step_ragged([None], [0], [21], prefix)
    (a,), sa, la = sess.step_ragged([p], [21], [1], [7], flags=pkg.RAGGED_SAMPLED | pkg.RAGGED_LOGITS)
    (b,), sb, lb = sess.step_ragged([p], [21], [1], [9], flags=pkg.RAGGED_SAMPLED | pkg.RAGGED_LOGITS)
    # reference replay: full sequences from scratch
    (ra,), _, rla = sess.step_ragged([None], [0], [22], np.append(prefix, 7), flags=pkg.RAGGED_LOGITS)
    (rb,), _, rlb = sess.step_ragged([None], [0], [22], np.append(prefix, 9), flags=pkg.RAGGED_LOGITS)
    # The replays' 22 tokens run the chunked-prefill attention kernel, the
    # branches' last token the split decode kernel: both round the softmax
    # weights to bf16, against different running maxima, so the last layer's
    # attention output (and the logits) differ at the 1e-4 level. The states
    # (KV rows, DeltaNet states) do not depend on that output.
    assert rel_l2(la[0], rla[0]) < 2e-3 and rel_l2(lb[0], rlb[0]) < 2e-3
    assert rel_l2(sess.snapshot(a), sess.snapshot(ra)) < 1e-4
    assert rel_l2(sess.snapshot(b), sess.snapshot(rb)) < 1e-4
    sess.release(p)
    (a2,), _, la2 = sess.step_ragged([a], [22], [1], [3], flags=pkg.RAGGED_LOGITS)
    (ra2,), _, rla2 = sess.step_ragged([ra], [22], [1], [3], flags=pkg.RAGGED_LOGITS)
    assert rel_l2(la2[0], rla2[0]) < 1e-4
    for o in (a, b, ra, rb, a2, ra2):
        sess.release(o)
    with pytest.raises(pkg.NativeError):
        sess.release(p)  # stale generation
    assert sess.stats()[0] == 0


def test_legacy_entry_points(tiny):
    """rs_qwen_device_step/_sampled/_block/_hidden_* and decode_batch agree with the ragged step."""
    pkg, cfg, store, sess, model = tiny
    toks = np.arange(5, dtype=np.uint32) * 31 + 3
    s1, l1 = sess.step(None, 0, toks)
    s2, tok = sess.step_sampled(None, 0, toks)
    s3, l3 = sess.step(None, 0, toks, block=True)
    s4, l4 = sess.step(None, 0, toks, hidden=True)
    assert tok == int(np.argmax(l1[0]))
    assert np.array_equal(l3[-1], l1[0]) and np.array_equal(l4[0], l1[0])
    h = sess.hidden_snapshot(s4, 5)
    assert h.shape == (5, cfg.hidden) and np.isfinite(h).all()
    outs, lb = sess.decode_batch([s1, s2], [11, 12])
    r1, _, rl = sess.step_ragged([s1, s2], [5, 5], [1, 1], [11, 12], flags=pkg.RAGGED_LOGITS)
    assert np.array_equal(lb, rl)
    for o in [s1, s2, s3, s4] + outs + r1:
        sess.release(o)


@pytest.fixture(scope="module")
def wide(pkg, O, cuda_ok):
    """configs[1] widths (hidden 2048, 512 experts top-10, 16q/2kv/256,
    GDN 32v/16qk/128, vocab 151936) cut to 4 layers so the FP64 oracle runs
    in seconds."""
    O.set_routing_slack(ROUTING_SLACK)
    cfg = pkg.config1(layers=4, context=4096)
    store = pkg.WeightStore().synthetic(cfg, SEED)
    sess = pkg.DeviceSession(store, cfg, slots=32, budget_bytes=8 << 30)
    model = O.Model(O.config1(layers=4, context=4096), SEED)
    yield pkg, cfg, store, sess, model
    sess.close()
    store.close()


def test_cfg1_width_decode_from_synthetic_state(wide):
    pkg, cfg, store, sess, model = wide
    positions = [37, 700, 2501]
    parents = [sess.synthetic_state(p, 77 + i) for i, p in enumerate(positions)]
    snaps = [sess.snapshot(p) for p in parents]
    toks = np.array([5, 151935, 70000], np.uint32)
    sess.set_capture(True)
    outs, sampled, logits = sess.step_ragged(parents, positions, [1, 1, 1], toks,
                                             flags=pkg.RAGGED_SAMPLED | pkg.RAGGED_LOGITS)
    route = sess.debug_routing(3)
    for s in range(3):
        lg, st, _, _ = model.forward([toks[s]], positions[s], old_state=snaps[s],
                                     forced_routing=route[:, s:s + 1, :])
        err = rel_l2(logits[s], lg[0])
        assert err < 1e-2, (s, err)
        assert rel_l2(sess.snapshot(outs[s]), st) < 1e-2
    for o in parents + outs:
        sess.release(o)


def test_cfg1_width_mixed_prefill_decode(wide):
    """configs[2] shape at configs[1] widths (4 layers): two prefill chunks and six
    decode tokens in one ragged step over synthetic prefix states.
    - EVERY row, each position along the 40- and 17-token chunks included,
      matches the FP64 oracle (fed the device's routing) within 1e-2. Along a
      chunk the recurrent state comes to hold only the step's own tokens, so
      the operand rounding of each projection accumulates into it; with fp16
      operands the oracle's emulation of that rounding puts the worst row at
      2.7e-3 (bf16 operands: 3.7e-2);
    - the chunks equal the same tokens decoded one step at a time (1e-3) up to
      the first router near-tie the two attention kernels resolve differently,
      and every one-token row matches the oracle fed its own routing (1e-2);
    - every sequence's logits equal, bit for bit, those of the sequence stepped
      alone (a token's arithmetic does not depend on the batch it is in)."""
    pkg, cfg, store, sess, model = wide
    rng = np.random.default_rng(31)
    positions = [100, 300, 37, 700, 2501, 64, 1000, 15]
    counts = [40, 17, 1, 1, 1, 1, 1, 1]
    parents = [sess.synthetic_state(p, 500 + i) for i, p in enumerate(positions)]
    snaps = [sess.snapshot(p) for p in parents]
    toks = [rng.integers(0, cfg.vocab, size=c).astype(np.uint32) for c in counts]
    flags = pkg.RAGGED_SAMPLED | pkg.RAGGED_LOGITS | pkg.RAGGED_ALL_ROWS
    sess.set_capture(True)
    outs, sampled, logits = sess.step_ragged(parents, positions, counts, np.concatenate(toks), flags=flags)
    route = sess.debug_routing(int(sum(counts)))
    sess.set_capture(False)
    cu = np.concatenate([[0], np.cumsum(counts)])
    for s in range(len(parents)):
        lg, st, _, _ = model.forward(toks[s], positions[s], old_state=snaps[s],
                                     forced_routing=route[:, cu[s]:cu[s + 1], :])
        errs = [rel_l2(logits[cu[s] + j], lg[j]) for j in range(counts[s])]
        assert max(errs) <= 1e-2, (s, [round(e, 5) for e in errs])
        assert rel_l2(sess.snapshot(outs[s]), st) < 1e-2, s
    for s in (0, 1):  # the chunks against one-token steps of the same tokens
        # The chunk's attention runs the prefill kernel, a one-token step the
        # split decode kernel (bf16 softmax weights against different maxima),
        # so a router near-tie can pick another expert; from then on the two
        # paths hold different (each valid) states. Rows before the first
        # divergence of the expert sets must agree within 1e-3; every
        # one-token row must match the oracle fed its own routing (1e-2).
        cur, step_logits, step_route, diverged = parents[s], [], [], None
        for j, t in enumerate(toks[s]):
            sess.set_capture(True)
            (nxt,), _, lj = sess.step_ragged([cur], [positions[s] + j], [1], [t], flags=pkg.RAGGED_LOGITS)
            rj = sess.debug_routing(1)
            sess.set_capture(False)
            if cur is not parents[s]:
                sess.release(cur)
            cur = nxt
            step_logits.append(lj[0])
            step_route.append(rj)
            same = all(set(rj[l, 0]) == set(route[l, cu[s] + j]) for l in range(cfg.layers))
            if diverged is None and not same:
                diverged = j
            if diverged is None:
                assert rel_l2(lj[0], logits[cu[s] + j]) < 1e-3, (s, j, rel_l2(lj[0], logits[cu[s] + j]))
        lg, st, _, _ = model.forward(toks[s], positions[s], old_state=snaps[s],
                                     forced_routing=np.concatenate(step_route, axis=1))
        errs = [rel_l2(step_logits[j], lg[j]) for j in range(counts[s])]
        assert max(errs) <= 1e-2, (s, [round(e, 5) for e in errs])
        if diverged is None:
            assert rel_l2(sess.snapshot(cur), sess.snapshot(outs[s])) < 1e-3, s
        assert rel_l2(sess.snapshot(cur), st) < 1e-2, s
        sess.release(cur)
    for s in range(len(parents)):
        (o1,), s1, l1 = sess.step_ragged([parents[s]], [positions[s]], [counts[s]], toks[s], flags=flags)
        assert np.array_equal(s1, sampled[cu[s]:cu[s + 1]])
        assert np.array_equal(l1, logits[cu[s]:cu[s + 1]]), s
        sess.release(o1)
    for o in parents + outs:
        sess.release(o)


def test_cfg1_width_long_prefill_runs(wide):
    """Runs of >= 64 tokens take the chunked DeltaNet kernels (64-token chunks,
    token-parallel conv preparation, the rows of each head's state carried
    chunk to chunk): a 100-token prefill from an empty state, a 64-token run
    and an 80-token run from synthetic prefix states, next to a decode row.
    Every row's logits and every sequence's state match the FP64 oracle (fed
    the device's routing) within 1e-2."""
    pkg, cfg, store, sess, model = wide
    rng = np.random.default_rng(77)
    positions = [0, 100, 900, 2000]
    counts = [100, 64, 80, 1]
    parents = [None] + [sess.synthetic_state(p, 800 + i) for i, p in enumerate(positions[1:])]
    snaps = [None] + [sess.snapshot(p) for p in parents[1:]]
    toks = [rng.integers(0, cfg.vocab, size=c).astype(np.uint32) for c in counts]
    flags = pkg.RAGGED_SAMPLED | pkg.RAGGED_LOGITS | pkg.RAGGED_ALL_ROWS
    sess.set_capture(True)
    outs, sampled, logits = sess.step_ragged(parents, positions, counts, np.concatenate(toks), flags=flags)
    route = sess.debug_routing(int(sum(counts)))
    sess.set_capture(False)
    cu = np.concatenate([[0], np.cumsum(counts)])
    for s in range(len(counts)):
        lg, st, _, _ = model.forward(toks[s], positions[s], old_state=snaps[s],
                                     forced_routing=route[:, cu[s]:cu[s + 1], :])
        errs = [rel_l2(logits[cu[s] + j], lg[j]) for j in range(counts[s])]
        assert max(errs) <= 1e-2, (s, max(errs), int(np.argmax(errs)))
        assert rel_l2(sess.snapshot(outs[s]), st) <= 1e-2, s
    for o in [p for p in parents if p is not None] + outs:
        sess.release(o)
