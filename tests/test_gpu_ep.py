"""Expert parallelism (rs_qwen_ep_unique_id / rs_qwen_device_ep_init): the
target model's MoE layers with the routed experts split over ranks, rows
exchanged with NCCL send/recv. A token's expert rows get the same arithmetic
as on one GPU, so the expert-parallel logits must equal the single-GPU
logits bit for bit.

- world = 1 (one GPU): the whole pack / plan / gather / return path runs with
  the self stage only;
- world = 2 (two GPUs, skipped otherwise): one process per GPU, each rank
  stepping its own sequences in lockstep, against a plain session of the same
  rank.
"""
import multiprocessing as mp
import os
import sys
from pathlib import Path

import numpy as np
import pytest

from conftest import has_cuda

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]


def _steps(pkg, cfg, sess, seed, n_seq):
    """A mixed prefill + decode step then a decode step on synthetic states;
    returns the sampled tokens and last-row logits of both steps."""
    rng = np.random.default_rng(seed)
    positions = [int(p) for p in rng.integers(5, 300, size=n_seq)]
    counts = [3] + [1] * (n_seq - 1)
    parents = [sess.synthetic_state(p, seed * 100 + i) for i, p in enumerate(positions)]
    toks = rng.integers(0, cfg.vocab, size=sum(counts)).astype(np.uint32)
    flags = pkg.RAGGED_SAMPLED | pkg.RAGGED_LOGITS
    outs, s1, l1 = sess.step_ragged(parents, positions, counts, toks, flags=flags)
    pos2 = [p + c for p, c in zip(positions, counts)]
    outs2, s2, l2 = sess.step_ragged(outs, pos2, [1] * n_seq, s1.astype(np.uint32), flags=flags)
    for o in parents + list(outs) + list(outs2):
        sess.release(o)
    return s1, l1, s2, l2


def _compare(pkg, cfg, store, world, rank, uid, seed, n_seq, exchange=None):
    """uid: NCCL transport; exchange(handle) -> all handles: direct NVLink stores
    (every rank then finishes its steps before any window is freed)."""
    plain = pkg.DeviceSession(store, cfg, slots=4 * n_seq, budget_bytes=2 << 30)
    ep = pkg.DeviceSession(store, cfg, slots=4 * n_seq, budget_bytes=2 << 30)
    if exchange is None:
        ep.ep_init(world, rank, uid, n_seq + 2)
    else:
        ep.ep_connect(exchange(ep.ep_window(world, rank, n_seq + 2)))
    try:
        a = _steps(pkg, cfg, plain, seed, n_seq)
        b = _steps(pkg, cfg, ep, seed, n_seq)
        if exchange is not None:
            exchange(b"done")
    finally:
        ep.close()
        plain.close()
    return all(np.array_equal(x, y) for x, y in zip(a, b))


@pytest.mark.parametrize("transport", ["nccl", "nvlink"])
@pytest.mark.parametrize("widths", ["cfg0", "cfg1"])
def test_expert_parallel_world1_equals_plain(pkg, widths, transport):
    if not has_cuda():
        pytest.skip("no CUDA device")
    cfg = pkg.config0() if widths == "cfg0" else pkg.config1(layers=4, context=1024)
    store = pkg.WeightStore().synthetic(cfg, 77)
    try:
        if transport == "nccl":
            assert _compare(pkg, cfg, store, 1, 0, pkg.ep_unique_id(), 5, 6)
        else:
            assert _compare(pkg, cfg, store, 1, 0, None, 5, 6, exchange=lambda h: [h] if h != b"done" else None)
    finally:
        store.close()


def _rank_main(rank, world, transport, qs, q_out):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    sys.path.insert(0, str(ROOT))
    import importlib
    import torch
    torch.cuda.set_device(rank)  # every GPU stays visible (peer windows)
    pkg = importlib.import_module("rust-ts-tokio-inference-engine_b200")
    try:
        def exchange(h):  # every rank's handle, in rank order
            for p in range(world):
                if p != rank:
                    qs[p].put((rank, h))
            got = {rank: h}
            while len(got) < world:
                r, hp = qs[rank].get(timeout=120)
                got[r] = hp
            return [got[p] for p in range(world)]
        uid = None
        if transport == "nccl":
            if rank == 0:
                uid = pkg.ep_unique_id()
                for p in range(1, world):
                    qs[p].put((0, uid))
            else:
                uid = qs[rank].get(timeout=120)[1]
        cfg = pkg.config1(layers=4, context=1024)
        store = pkg.WeightStore().synthetic(cfg, 77)
        ok = _compare(pkg, cfg, store, world, rank, uid, 11 + rank, 5,
                      exchange=exchange if transport == "nvlink" else None)
        q_out.put((rank, bool(ok), ""))
        store.close()
    except Exception as e:  # reported to the parent; never left hanging
        q_out.put((rank, False, repr(e)))


@pytest.mark.parametrize("transport", ["nccl", "nvlink"])
def test_expert_parallel_two_gpus_equals_plain(transport):
    import torch
    if not has_cuda() or torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    qs, q_out = [ctx.Queue() for _ in range(2)], ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, transport, qs, q_out)) for r in range(2)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in range(2):
            r, ok, msg = q_out.get(timeout=600)
            results[r] = (ok, msg)
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    assert results == {0: (True, ""), 1: (True, "")}, results
