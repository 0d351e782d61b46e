"""Host logic of multi-GPU launches on CPU: program-range sharding and the
gather of output shards, with world size 2 over gloo (the GPU path uses the
same code over NCCL)."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from tila_b200.multigpu import gather_leading, shard_range, shard_rows


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


def test_shard_rows_follow_the_program_split():
    # 3 matmul tile rows of 128 on 2 GPUs: programs [0, 2) and [2, 3)
    assert shard_rows(3, 128, 384, 2) == [(0, 256), (256, 384)]
    # a ragged last program (rows 300 of 3 tiles) and more ranks than programs
    assert shard_rows(3, 128, 300, 2) == [(0, 256), (256, 300)]
    assert shard_rows(2, 128, 256, 3) == [(0, 128), (128, 256), (256, 256)]
    with pytest.raises(ValueError):
        shard_rows(2, 128, 384, 2)


def _worker(rank, world, port, rows, q, per_program=None):
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank,
                            world_size=world)
    try:
        out = torch.full((rows, 3), -1.0)
        ranges = None
        if per_program is None:
            lo, hi = shard_range(rows, world, rank)
        else:
            ranges = shard_rows(-(-rows // per_program), per_program, rows, world)
            lo, hi = ranges[rank]
        out[lo:hi] = torch.arange(lo, hi, dtype=torch.float32)[:, None] * 10 + torch.arange(3)
        gather_leading(out, world, rank, rows=ranges)
        expected = torch.arange(rows, dtype=torch.float32)[:, None] * 10 + torch.arange(3)
        q.put((rank, bool(torch.equal(out, expected))))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("rows,per_program", [(10, None), (11, None), (384, 128), (300, 128)])
def test_gather_of_output_shards_world2(rows, per_program):
    """Rows written by each rank's programs are gathered, including uneven
    program splits whose row shards differ from a split of the rows (3 tile
    rows of 128: ranks write 256 and 128 rows)."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, rows, q, per_program)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    results = dict(q.get(timeout=10) for _ in range(2))
    assert results == {0: True, 1: True}
