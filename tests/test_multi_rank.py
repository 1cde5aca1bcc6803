"""bench.py's multi-rank plumbing on CPU: two gloo ranks (the GPU ranks use
NCCL with the same calls). Each rank contributes its own device time; the
reported time must be the maximum over ranks on every rank, and the barrier
must hold both ranks."""
import os
import socket
import sys
import time
from pathlib import Path

import pytest
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, out):
    os.environ.update(RANK=str(rank), WORLD_SIZE=str(world), LOCAL_RANK=str(rank), MASTER_ADDR="127.0.0.1",
                      MASTER_PORT=str(port))
    sys.path.insert(0, str(ROOT))
    import bench
    r, w, local = bench.dist_setup(world)
    assert (r, w, local) == (rank, world, rank)
    if rank == 1:
        time.sleep(0.5)  # the barrier must wait for the slow rank
    t0 = time.perf_counter()
    bench.barrier(w)
    waited = time.perf_counter() - t0
    m = bench.max_over_ranks(1.25 + rank, w)
    out.put((rank, m, waited))
    import torch.distributed as dist
    dist.destroy_process_group()


def test_two_gloo_ranks_time_is_max_over_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = sorted(q.get(timeout=5) for _ in range(2))
    assert [r[1] for r in res] == [2.25, 2.25]
    assert res[0][2] >= 0.3  # rank 0 waited for rank 1 at the barrier


def test_world_size_must_match_gpus(monkeypatch):
    sys.path.insert(0, str(ROOT))
    import bench
    monkeypatch.setenv("WORLD_SIZE", "2")
    monkeypatch.setenv("RANK", "0")
    with pytest.raises(SystemExit):
        bench.dist_setup(4)
