"""Multi-rank logic of the data-parallel benchmark on CPU (gloo, world size 2).

Each rank processes its own observations (no collective in the data path);
the only cross-rank steps are the timing barrier and the max-over-ranks of the
step time, which set the whole-job throughput.
"""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import bench


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        # rank r pretends its step took 2 + r ms
        ms = bench.max_over_ranks(2.0 + rank, torch.device("cpu"))
        dist.barrier()
        out[rank] = (ms, bench.job_throughput(ms, per_rank_prefixes=3, world=world))
    finally:
        dist.destroy_process_group()


def test_max_over_ranks_and_weak_scaling_throughput():
    world = 2
    with mp.Manager() as mgr:
        out = mgr.dict()
        mp.spawn(_worker, args=(world, _free_port(), out), nprocs=world, join=True)
        res = dict(out)
    # every rank sees the slowest rank's time
    assert res[0][0] == res[1][0] == 3.0
    # 3 observations per rank x 2 ranks in 3 ms
    assert res[0][1] == pytest.approx(2000.0)


def test_single_rank_throughput():
    assert bench.job_throughput(4.0, 1, 1) == pytest.approx(250.0)
