"""Host logic of multi-GPU launches on CPU: program-range sharding and the
gather of output shards, with world size 2 over gloo (the GPU path uses the
same code over NCCL)."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from tila_b200.multigpu import gather_leading, shard_range


@pytest.mark.parametrize("total,world", [(8192, 2), (7, 2), (128, 8), (1, 4), (0, 3)])
def test_shard_ranges_partition_the_grid(total, world):
    ranges = [shard_range(total, world, r) for r in range(world)]
    assert ranges[0][0] == 0 and ranges[-1][1] == total
    for (a, b), (c, d) in zip(ranges, ranges[1:]):
        assert b == c and b - a >= d - c
    assert max(b - a for a, b in ranges) - min(b - a for a, b in ranges) <= 1


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, rows, q):
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    try:
        out = torch.full((rows, 3), -1.0)
        lo, hi = shard_range(rows, world, rank)
        out[lo:hi] = torch.arange(lo, hi, dtype=torch.float32)[:, None] * 10 + torch.arange(3)
        gather_leading(out, world, rank)
        expected = torch.arange(rows, dtype=torch.float32)[:, None] * 10 + torch.arange(3)
        q.put((rank, bool(torch.equal(out, expected))))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("rows", [10, 11])
def test_gather_of_output_shards_world2(rows):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, rows, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    results = dict(q.get(timeout=10) for _ in range(2))
    assert results == {0: True, 1: True}
