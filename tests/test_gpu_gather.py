"""The C-ABI NCCL gather (tila_mg_*) on the GPU.  One rank here; the
two-to-eight-rank path runs in ``bench.py --gpus N`` (the output rows each
rank computed are gathered through the same communicator)."""

import pytest

import tila_b200
from tila_b200 import multigpu

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


def test_single_rank_gather_copies_the_shard():
    comm = multigpu.Communicator(1, 0, torch.device("cuda", 0))
    try:
        send = torch.arange(1000, dtype=torch.float32, device="cuda")
        recv = torch.full((1000,), -1.0, device="cuda")
        comm.all_gather(send, recv)
        torch.cuda.synchronize()
        assert torch.equal(recv, send)
        out = torch.randn(37, 5, device="cuda")
        ref = out.clone()
        multigpu.gather_leading(out, 1, 0, comm=comm)
        torch.cuda.synchronize()
        assert torch.equal(out, ref)
    finally:
        comm.close()
    assert tila_b200.read_device_errors() == 0
