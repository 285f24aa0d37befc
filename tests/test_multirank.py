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


# ----------------------------------------------------------------------------- sharded MLP
def _shard_worker(rank: int, world: int, port: int, out):
    from pi05_pytorch_fast_b200.shard import MlpShard, exchange_row_blocks, gather_row_blocks

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        sh = MlpShard(rank, world)
        m, n, hidden = 12, 64, 8
        gen = torch.Generator().manual_seed(5)
        h = torch.randn(m, n, generator=gen)          # the full GeGLU output, same on every rank
        w = torch.randn(hidden, n, generator=gen, dtype=torch.float64)
        part = h[:, sh.cols(n)].contiguous()          # what this rank's gate/up shard produces
        seg = n // world
        recv = torch.empty(world, m // world, seg)
        exchange_row_blocks(part, recv, sh)
        mine = m // world
        # the addressing w4a4_quant_segments documents: element e of row r at
        # (e / seg) * seg_stride + r * ld + e % seg, ld = seg, seg_stride = mine * seg
        flat = recv.view(-1)
        e = torch.arange(n)
        rows = torch.stack([flat[(e // seg) * (mine * seg) + r * seg + e % seg] for r in range(mine)])
        ok_rows = torch.equal(rows, h[sh.rows(m)])
        y_part = rows.double() @ w.T                  # down_proj of this rank's rows
        y = torch.empty(m, hidden, dtype=torch.float64)
        gather_row_blocks(y_part, y, sh)
        ok_y = torch.allclose(y, h.double() @ w.T, rtol=0, atol=1e-12)
        out[rank] = (ok_rows, ok_y)
    finally:
        dist.destroy_process_group()


def test_sharded_mlp_exchange_and_gather_rebuild_the_full_rows():
    world = 2
    with mp.Manager() as mgr:
        out = mgr.dict()
        mp.spawn(_shard_worker, args=(world, _free_port(), out), nprocs=world, join=True)
        res = dict(out)
    assert res == {0: (True, True), 1: (True, True)}


def test_mlp_shard_slices():
    from pi05_pytorch_fast_b200.shard import MlpShard

    sh = MlpShard(2, 4)
    assert sh.cols(16384) == slice(8192, 12288) and sh.rows(776) == slice(388, 582)
    with pytest.raises(ValueError, match="not divisible"):
        MlpShard(0, 3).rows(776)
