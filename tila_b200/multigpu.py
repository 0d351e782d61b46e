"""Multi-GPU launches: split a kernel's program grid across GPUs.

Programs of a Tila kernel are independent, so a launch shards by giving
each rank (one process per GPU) a contiguous range of ``program_id`` values
along one grid axis.  Every rank runs the full launch contract and proofs on
the full grid (``kernel[grid](...)`` unchanged) while only its programs
execute; ``program_id`` and ``num_programs`` keep their global values.  The
rows of the output that a rank's programs wrote are then gathered with NCCL
over NVLink (``torch.distributed``), the only collective on this path.
"""

from __future__ import annotations

from contextlib import contextmanager

from .backend import program_range


def shard_range(total: int, world: int, rank: int):
    """Contiguous [lo, hi) share of ``total`` programs for ``rank``; the
    first ``total % world`` ranks get one extra program."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("rank must be in [0, world)")
    base, extra = divmod(int(total), world)
    lo = rank * base + min(rank, extra)
    hi = lo + base + (1 if rank < extra else 0)
    return lo, hi


@contextmanager
def shard(axis: int, total: int, world: int, rank: int):
    """Inside the block, B200 launches run only this rank's programs along
    ``axis`` (of ``total`` programs)."""
    lo, hi = shard_range(total, world, rank)
    with program_range(axis, lo, hi):
        yield lo, hi


class Communicator:
    """NCCL communicator of the ranks' GPUs behind the C ABI (``tila_mg_*``):
    rank 0 creates the id, ``torch.distributed`` (any backend) carries it to
    the other ranks, and every rank joins on its current device."""

    def __init__(self, world: int, rank: int, device, group=None):
        import torch
        import torch.distributed as dist
        from . import native
        box = [native.mg_unique_id() if rank == 0 else None]
        if world > 1:
            dist.broadcast_object_list(box, src=0, group=group)
        with torch.cuda.device(device):
            self.handle = native.mg_comm_init(box[0], world, rank)
        self.world, self.rank, self.device = world, rank, device

    def all_gather(self, send, recv):
        """recv (world x send.numel() elements, contiguous) = every rank's send,
        in rank order, on the current stream."""
        import torch
        from . import native
        if not (send.is_contiguous() and recv.is_contiguous()):
            raise ValueError("gather buffers must be contiguous")
        nbytes = send.numel() * send.element_size()
        if recv.numel() * recv.element_size() != nbytes * self.world:
            raise ValueError("receive buffer must hold world x send bytes")
        stream = torch.cuda.current_stream(self.device).cuda_stream
        native.mg_gather(self.handle, send.data_ptr(), recv.data_ptr(), nbytes, stream)

    def close(self):
        from . import native
        if self.handle:
            native.mg_comm_destroy(self.handle)
            self.handle = None


def shard_rows(programs: int, rows_per_program: int, rows: int, world: int):
    """Leading-dimension rows of the output that each rank's programs write
    when ``programs`` programs of the sharded axis are split by
    :func:`shard_range` and program p writes rows
    ``[p * rows_per_program, (p + 1) * rows_per_program)`` (clipped to
    ``rows``): one per rank, contiguous, covering ``[0, rows)``.  Example: 3
    matmul tile rows of 128 on 2 GPUs -> programs [0, 2) and [2, 3) -> rows
    [0, 256) and [256, 384)."""
    out = []
    for r in range(world):
        lo, hi = shard_range(programs, world, r)
        out.append((min(lo * rows_per_program, rows), min(hi * rows_per_program, rows)))
    if out and (out[0][0] != 0 or out[-1][1] != rows):
        raise ValueError(f"{programs} programs of {rows_per_program} rows do not cover {rows} rows")
    return out


def gather_leading(out, world: int, rank: int, rows=None, group=None, comm: Communicator = None):
    """All-gather the leading-dimension shards of ``out`` in place.

    ``rows[r]`` is the ``[lo, hi)`` range of leading rows that rank r wrote
    (:func:`shard_rows` computes it from the program split); the ranges are
    contiguous, in rank order, and cover ``out``.  Without ``rows`` the rows
    are split by :func:`shard_range` (right when each program of the sharded
    axis writes one leading row).  After the call every rank holds the full
    tensor.  With ``comm`` (the C-ABI NCCL communicator), a contiguous ``out``
    and equal shards, the ranks' shards are gathered straight into ``out``
    (each rank's own rows are its send buffer); otherwise shards are padded
    to the largest one for the collective, which runs through ``comm`` or
    ``torch.distributed``.
    """
    import torch
    import torch.distributed as dist
    n = out.shape[0]
    ranges = [tuple(r) for r in rows] if rows is not None else [shard_range(n, world, r) for r in range(world)]
    if len(ranges) != world or ranges[0][0] != 0 or ranges[-1][1] != n or \
            any(b != c for (_, b), (c, _) in zip(ranges, ranges[1:])) or any(b < a for a, b in ranges):
        raise ValueError(f"row ranges {ranges} do not partition {n} rows over {world} ranks")
    sizes = [b - a for a, b in ranges]
    lo, hi = ranges[rank]
    if comm is not None and out.is_contiguous() and len(set(sizes)) == 1:
        comm.all_gather(out[lo:hi], out)
        return out
    width = max(sizes)
    send = torch.empty((width,) + tuple(out.shape[1:]), dtype=out.dtype, device=out.device)
    send[: hi - lo] = out[lo:hi]
    if comm is not None:
        flat = torch.empty((world,) + tuple(send.shape), dtype=out.dtype, device=out.device)
        comm.all_gather(send, flat)
        recv = list(flat.unbind(0))
    else:
        recv = [torch.empty_like(send) for _ in range(world)]
        dist.all_gather(recv, send, group=group)
    for r, (a, b) in enumerate(ranges):
        if r != rank and b > a:
            out[a:b] = recv[r][: b - a]
    return out
