"""Bit-exact integer outputs of the CUDA path against the oracle's rules on
identical inputs: top-k expert ids given the device's router logits, the
stable token->expert sort (offsets, permutation), and ragged packing
(prefix sums, per-token positions, KV slots, child block-table rows)."""
import numpy as np
import pytest

from conftest import has_cuda

pytestmark = pytest.mark.gpu

SEQ_DESC_INTS = 13  # SeqDesc: position, count, parent, child, n_shared, new_off, n_new, out_row0, n_out, cow_src, cow_len, hidden, cand


@pytest.fixture(scope="module")
def wide(pkg, O):
    if not has_cuda():
        pytest.skip("no CUDA device")
    cfg = pkg.config1(layers=4, context=2048)
    store = pkg.WeightStore().synthetic(cfg, 5)
    sess = pkg.DeviceSession(store, cfg, slots=160, budget_bytes=16 << 30)
    yield pkg, cfg, store, sess
    sess.close()
    store.close()


def _decode_batch(pkg, sess, cfg, n, seed):
    rng = np.random.default_rng(seed)
    pos = rng.integers(1, 1500, size=n)
    parents = [sess.synthetic_state(int(p), seed + i) for i, p in enumerate(pos)]
    toks = rng.integers(0, cfg.vocab, size=n).astype(np.uint32)
    sess.set_capture(True)
    outs, sampled, _ = sess.step_ragged(parents, pos, np.ones(n, np.uint32), toks)
    return parents, outs


def test_topk_and_sort_bit_exact(wide, O):
    pkg, cfg, store, sess = wide
    sess.drain()
    n, E, K = 64, cfg.experts, cfg.top
    parents, outs = _decode_batch(pkg, sess, cfg, n, 11)
    logits = sess.debug_capture(0, np.float32).reshape(cfg.layers, n, E + 1)
    offsets = sess.debug_capture(1).reshape(cfg.layers, E + 2)
    perm = sess.debug_capture(2).reshape(cfg.layers, n * (K + 1))
    ids = sess.debug_routing(n)
    for layer in range(cfg.layers):
        mine = O.topk(logits[layer, :, :E], K)
        assert np.array_equal(mine, ids[layer]), layer
        flat = np.concatenate([ids[layer], np.full((n, 1), E, np.int32)], axis=1).ravel()
        counts, offs, p, inv = O.expert_sort(flat, E + 1)
        assert np.array_equal(offs, offsets[layer, : E + 2]), layer
        assert np.array_equal(p, perm[layer]), layer
    # the captured selection is a valid top-k of the captured logits and its
    # renormalised weights follow operator_reference.h:47-57
    import ctypes as C
    for layer in range(cfg.layers):
        probs, w = np.zeros(n * E), np.zeros(n * K)
        lg = np.ascontiguousarray(logits[layer, :, :E])
        sel = np.ascontiguousarray(ids[layer])
        O.call("orc_routing", O.ptr(lg), O.ptr(sel, C.c_int32), n, E, K, O.ptr(probs, C.c_double),
               O.ptr(w, C.c_double))
    sess.drain()


@pytest.mark.parametrize("T", [200, 256, 300])
def test_prefill_routing_sort_bit_exact(wide, O, T):
    """Prefill-sized steps (the chunked-prefill attention and DeltaNet kernels
    upstream of the router): top-k ids given the captured router logits and
    the stable expert sort equal the oracle's rules, layer by layer."""
    pkg, cfg, store, sess = wide
    sess.drain()
    E, K = cfg.experts, cfg.top
    toks = np.random.default_rng(T).integers(0, cfg.vocab, size=T).astype(np.uint32)
    sess.set_capture(True)
    outs, _, _ = sess.step_ragged([None], [0], [T], toks)
    logits = sess.debug_capture(0, np.float32).reshape(cfg.layers, T, E + 1)
    offsets = sess.debug_capture(1).reshape(cfg.layers, E + 2)
    perm = sess.debug_capture(2).reshape(cfg.layers, T * (K + 1))
    ids = sess.debug_routing(T)
    sess.set_capture(False)
    for layer in range(cfg.layers):
        assert np.array_equal(O.topk(logits[layer, :, :E], K), ids[layer]), layer
        flat = np.concatenate([ids[layer], np.full((T, 1), E, np.int32)], axis=1).ravel()
        counts, offs, p, inv = O.expert_sort(flat, E + 1)
        assert np.array_equal(offs, offsets[layer, : E + 2]), layer
        assert np.array_equal(p, perm[layer]), layer
    sess.release(outs[0])
    sess.drain()


def _unpack(blob):
    n, T, R, nn = map(int, blob[:4])
    o = 4
    descs = blob[o:o + n * SEQ_DESC_INTS].reshape(n, SEQ_DESC_INTS)
    o += n * SEQ_DESC_INTS
    pages = blob[o:o + nn]
    o += nn
    cu = blob[o:o + n + 1]
    o += n + 1
    tseq = blob[o:o + T]
    o += T
    tpos = blob[o:o + T]
    o += T
    slots = blob[o:o + T]
    o += T
    out_tok = blob[o:o + R]
    return n, T, R, descs, pages, cu, tseq, tpos, slots, out_tok


def test_packing_bit_exact(wide, O):
    """Prefill 5 ragged prompts, then a mixed step: decode, a second chunk, and
    two branches of one parent (copy-on-write of a shared partial page)."""
    pkg, cfg, store, sess = wide
    sess.drain()
    sess.set_capture(True)
    rng = np.random.default_rng(2)
    lens = np.array([3, 16, 17, 40, 1], np.uint32)
    toks = rng.integers(0, cfg.vocab, size=int(lens.sum())).astype(np.uint32)
    outs1, _, _ = sess.step_ragged([None] * 5, [0] * 5, lens, toks)
    blob1 = sess.debug_capture(3)
    rows1 = sess.debug_capture(4)
    n1, T1, R1, d1, pages1, *_ = _unpack(blob1)
    maxp1 = rows1.size // n1
    bt = np.full((160, 2048 // 16 + 1), -7, np.int32)
    for i in range(n1):
        np_i = int(d1[i, 4] + d1[i, 6])
        bt[d1[i, 3], :np_i] = rows1.reshape(n1, maxp1)[i, :np_i]
    parents = [outs1[0], outs1[1], outs1[2], outs1[2], outs1[3]]
    pos = np.array([3, 16, 17, 17, 40], np.uint32)
    cnt = np.array([1, 20, 1, 2, 1], np.uint32)
    toks2 = rng.integers(0, cfg.vocab, size=int(cnt.sum())).astype(np.uint32)
    outs2, _, _ = sess.step_ragged(parents, pos, cnt, toks2, flags=pkg.RAGGED_SAMPLED | pkg.RAGGED_ALL_ROWS)
    blob2 = sess.debug_capture(3)
    rows2 = sess.debug_capture(4)
    n, T, R, d, pages, cu, tseq, tpos, slots, out_tok = _unpack(blob2)
    assert n == 5 and T == int(cnt.sum()) and R == T
    assert d[3, 9] >= 0, "second branch of a shared partial page must copy on write"
    cu_o, tseq_o, tpos_o, slots_o, bt_o = O.pack_ragged(
        d[:, 0], d[:, 1], d[:, 2], d[:, 3], d[:, 4], d[:, 5], d[:, 6], pages, 16, bt)
    assert np.array_equal(cu, cu_o)
    assert np.array_equal(tseq, tseq_o)
    assert np.array_equal(tpos, tpos_o)
    assert np.array_equal(slots, slots_o.astype(np.int32))
    maxp = rows2.size // n
    for i in range(n):
        np_i = int(d[i, 4] + d[i, 6])
        assert np.array_equal(rows2.reshape(n, maxp)[i, :np_i], bt_o[d[i, 3], :np_i]), i
    # every output row is the token itself (ALL_ROWS)
    assert np.array_equal(out_tok, np.arange(T, dtype=np.int32))
    sess.drain()
