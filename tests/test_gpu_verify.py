"""Device speculative verify + accept (rs_qwen_device_mtp_verify_accept).

Against the plain greedy path on the same parents: for each sequence the
target is stepped one token at a time from the parent ([seed, r_0, r_1, ...],
r_j the greedy token after fed token j), which gives the rows the accept rule
sees and the version after every prefix. The verify call must then report
the accepted count and emitted tokens of the reference's plan() rule (the
oracle's orc_accept, pinned to src/serving/native_speculative.rs's cases)
bit-exactly, and its output version must equal the replayed version after
[seed, d_0 .. d_{accepted-1}] bit-for-bit: KV, DeltaNet state, conv history
(the snapshot) and the kept hidden rows. Runs at configs[0] and at
configs[1] widths.
"""
import numpy as np
import pytest

from conftest import has_cuda

pytestmark = pytest.mark.gpu

K = 4  # drafts of the longest sequence


def greedy_chain(pkg, sess, parent, pos, seed, steps):
    """Versions after [seed], [seed, r_0], ... and the rows r_0 .. r_{steps-1}."""
    versions, rows, hidden = [], [], []
    cur, tok = parent, seed
    for j in range(steps):
        outs, s, _ = sess.step_ragged([cur], [pos + j], [1], [tok], flags=pkg.RAGGED_SAMPLED | pkg.RAGGED_HIDDEN)
        versions.append(outs[0])
        hidden.append(sess.hidden_snapshot(outs[0], 1)[0])
        rows.append(int(s[0]))
        cur, tok = outs[0], int(s[0])
    return versions, rows, hidden


@pytest.fixture(scope="module", params=["cfg0", "cfg1"])
def setup(pkg, request):
    """configs[0], and configs[1] widths on a 4-layer slice."""
    if not has_cuda():
        pytest.skip("no CUDA device")
    cfg = pkg.config0() if request.param == "cfg0" else pkg.config1(layers=4, context=1024)
    store = pkg.WeightStore().synthetic(cfg, 7)
    sess = pkg.DeviceSession(store, cfg, slots=96, budget_bytes=4 << 30)
    rng = np.random.default_rng(11)
    lens = [5, 9, 3, 12, 7]
    prompts = [rng.integers(0, cfg.vocab, size=n).astype(np.uint32) for n in lens]
    outs, seeds, _ = sess.step_ragged([None] * len(lens), [0] * len(lens), lens, np.concatenate(prompts),
                                      flags=pkg.RAGGED_SAMPLED)
    chains = [greedy_chain(pkg, sess, outs[i], lens[i], int(seeds[i]), K + 1) for i in range(len(lens))]
    yield cfg, sess, outs, [int(x) for x in seeds], lens, chains
    sess.close()
    store.close()


def test_verify_accept_matches_plan_and_replay(pkg, O, setup):
    cfg, sess, parents, seeds, lens, chains = setup
    rows = [c[1] for c in chains]
    wrong = lambda t: (t + 1) % cfg.vocab
    drafts = [
        rows[0][:K],                                       # all accepted: bonus r_K
        [wrong(rows[1][0])] + rows[1][1:K],                # rejected at once
        rows[2][:2] + [wrong(rows[2][2])] + rows[2][3:K],  # two accepted
        [],                                                # no drafts: the seed's row is the bonus
        rows[4][:3],                                       # all of a shorter draft accepted
    ]
    outs, acc, emitted = sess.verify_accept(parents, seeds, drafts, flags=pkg.RAGGED_HIDDEN)
    for i in range(len(parents)):
        remaining = cfg.context - lens[i] - 1
        em_ref, acc_ref, _ = O.accept(rows[i][0], drafts[i], rows[i][1:len(drafts[i]) + 1], [], remaining)
        assert acc[i] == acc_ref and emitted[i] == em_ref, (i, acc[i], acc_ref, emitted[i], em_ref)
        ref = chains[i][0][acc[i]]
        assert outs[i].position == lens[i] + 1 + acc[i] == ref.position
        assert np.array_equal(sess.snapshot(outs[i]), sess.snapshot(ref)), i
        hid = sess.hidden_snapshot(outs[i], acc[i] + 1)
        assert np.array_equal(hid, np.stack(chains[i][2][:acc[i] + 1])), i


def test_verify_accept_stops_at_eos(pkg, O, setup):
    cfg, sess, parents, seeds, lens, chains = setup
    rows = chains[1][1]
    eos = [rows[1]]
    drafts = [rows[:K]]
    outs, acc, emitted = sess.verify_accept([parents[1]], [seeds[1]], drafts, eos=eos)
    em_ref, acc_ref, term = O.accept(rows[0], drafts[0], rows[1:K + 1], eos, cfg.context - lens[1] - 1)
    assert term and acc[0] == acc_ref and emitted[0] == em_ref
    assert np.array_equal(sess.snapshot(outs[0]), sess.snapshot(chains[1][0][acc[0]]))


def test_verify_accept_rejects_bad_geometry(pkg, setup):
    cfg, sess, parents, seeds, lens, chains = setup
    with pytest.raises(pkg.NativeError):
        sess.verify_accept([parents[0]], [seeds[0]], [[1] * 9])  # more than 8 drafts
