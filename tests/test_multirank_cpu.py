"""bench.py's multi-rank host logic on CPU: two gloo ranks (world size 2).

Covers what the multi-GPU bench relies on besides the kernels: rank/world
from the environment, the barrier, and the max-over-ranks of the step time
(the slowest rank defines the job's time), the per-rank breakdown every rank
gathers, and that the whole-job value sums the work of all ranks over that
time.
"""
from __future__ import annotations

import os
import socket

import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out):
    os.environ.update({"RANK": str(rank), "LOCAL_RANK": str(rank), "WORLD_SIZE": str(world),
                       "MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port)})
    import bench
    import torch.distributed as dist
    w, r, local = bench.init_dist()
    assert (w, r, local) == (world, rank, rank)
    bench.barrier(w)
    step_ms = 1.0 + rank            # rank 1 is the slow one
    worst = bench.max_over_ranks(step_ms, w, "cpu")
    rows = bench.gather_rows([step_ms, 10.0 * rank], w, "cpu")   # per-rank breakdown
    out[rank] = (worst, rows)
    dist.destroy_process_group()


def test_two_gloo_ranks_max_over_ranks():
    world = 2
    port = _free_port()
    with mp.Manager() as m:
        out = m.dict()
        mp.spawn(_worker, args=(world, port, out), nprocs=world, join=True)
        expect = (2.0, [[1.0, 0.0], [2.0, 10.0]])
        assert dict(out) == {0: expect, 1: expect}
