"""tila_launch_noalloc: the launch entry point for callers that cannot
allocate device memory.

Callers that record CUDA graphs, that run inside a host whose own pool owns
all device memory, or that cannot afford cudaMalloc's synchronisation in a
hot loop cannot provide the per-launch scratch word (the error word) that
tila_launch expects.  tila_launch_noalloc takes the same kernel and arguments
and substitutes a static device array owned by the library.  This test runs a
generated kernel through it twice in a row, through the C ABI, and checks each
output against the output of the normal entry point.
"""

import ctypes

import numpy as np
import pytest
import torch

import tila_b200
from tila_b200 import native, workloads as W
from tila_b200.backend import last_launch

pytestmark = pytest.mark.gpu


def test_noalloc_launch_matches_normal_entry_point():
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    x = torch.from_numpy(W.softmax_inputs(256, 1000, seed=41)).to(dev)
    reference = torch.zeros_like(x)
    W.row_softmax[(256,)](x, reference, BN=1024)          # normal entry point
    torch.cuda.synchronize()
    rec = last_launch(W.row_softmax)
    params = rec.entry.spec.params
    out_index = next(i for i, p in enumerate(params) if p[0] == "buffer" and p[1] == "o")
    err_index = next(i for i, p in enumerate(params) if p[0] == "err")
    stream = torch.cuda.current_stream(dev).cuda_stream
    for call in range(2):
        out = torch.full_like(x, float("nan"))
        args = list(rec.args)
        args[out_index] = ctypes.c_uint64(out.data_ptr())
        status = rec.entry.kernel.launch_noalloc(rec.grid, (rec.entry.spec.threads, 1, 1), args,
                                                 err_index, 4, smem_bytes=rec.entry.spec.smem_bytes,
                                                 stream=stream)
        assert status == native.TILA_OK, rec.entry.kernel.last_log
        torch.cuda.synchronize()
        np.testing.assert_allclose(out.cpu().numpy(), reference.cpu().numpy(), rtol=1e-6, atol=0)


def test_noalloc_rejects_scratch_beyond_its_capacity():
    dev = torch.device("cuda", 0)
    x = torch.from_numpy(W.softmax_inputs(8, 1000, seed=42)).to(dev)
    o = torch.zeros_like(x)
    W.row_softmax[(8,)](x, o, BN=1024)
    rec = last_launch(W.row_softmax)
    err_index = next(i for i, p in enumerate(rec.entry.spec.params) if p[0] == "err")
    status = rec.entry.kernel.launch_noalloc(rec.grid, (rec.entry.spec.threads, 1, 1), list(rec.args),
                                             err_index, native.NOALLOC_SCRATCH_BYTES + 1,
                                             smem_bytes=rec.entry.spec.smem_bytes)
    assert status == native.TILA_ERR_ARGUMENT
    assert "at most" in rec.entry.kernel.last_log
