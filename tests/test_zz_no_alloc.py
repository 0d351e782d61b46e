"""tila_launch_noalloc: the launch entry point for callers that cannot
allocate device memory.

Some hosts own every byte of device memory through their own pool and forbid
the CUDA allocator; some loops cannot afford cudaMalloc's implicit device
synchronisation.  Neither can provide the per-launch scratch block (the
kernel's error block) that tila_launch expects.  tila_launch_noalloc takes
the same kernel and arguments and substitutes a static device array owned by
the library, and tila_noalloc_read_error reads what a launch recorded there.

The tests call both through the C ABI: a generated kernel twice in a row,
each output equal to the normal entry point's bit for bit; a launch whose
bounded wait times out records its code and line in the static scratch, and
the next launch starts from a cleared word; scratch requests beyond the
array's capacity are rejected.  This file is collected last on purpose.
"""

import ctypes

import numpy as np
import pytest
import torch

import tila_b200
from tila_b200 import native, workloads as W
from tila_b200.backend import last_launch

pytestmark = pytest.mark.gpu


def _softmax_record(dev, rows, seed):
    x = torch.from_numpy(W.softmax_inputs(rows, 1000, seed=seed)).to(dev)
    reference = torch.zeros_like(x)
    W.softmax_kernel[(rows,)](x, reference, BN=1024)          # normal entry point
    torch.cuda.synchronize()
    return x, reference, last_launch(W.softmax_kernel)


def _noalloc(rec, args, scratch_bytes, stream):
    spec = rec.entry.spec
    err_index = next(i for i, p in enumerate(spec.params) if p[0] == "err")
    return rec.entry.kernel.launch_noalloc(rec.grid, (spec.threads, 1, 1), args, err_index,
                                           scratch_bytes, smem_bytes=spec.smem_bytes, stream=stream)


def test_noalloc_launch_matches_normal_entry_point():
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    x, reference, rec = _softmax_record(dev, 256, 41)
    out_index = next(i for i, p in enumerate(rec.entry.spec.params) if p[0] == "buffer" and p[1] == "o")
    stream = torch.cuda.current_stream(dev).cuda_stream
    for call in range(2):
        out = torch.full_like(x, float("nan"))
        args = list(rec.args)
        args[out_index] = ctypes.c_uint64(out.data_ptr())
        status = _noalloc(rec, args, native.ERROR_BLOCK_BYTES, stream)
        assert status == native.TILA_OK, rec.entry.kernel.last_log
        torch.cuda.synchronize()
        np.testing.assert_array_equal(out.cpu().numpy(), reference.cpu().numpy())
        assert native.noalloc_read_error(stream) == 0


PROBE = r'''
#include "tila_tile.cuh"
extern "C" __global__ void tila_noalloc_wait_probe(tila::u32 *err) {
  __shared__ __align__(8) tila::u64 bar;
  __shared__ int dead;
  if (threadIdx.x == 0) { tila::mbar_init(&bar, 1); dead = 0; tila::mbar_fence_init(); }
  __syncthreads();
  if (threadIdx.x == 0) tila::mbar_wait(&bar, 0u, err, 777u, &dead);
}
'''


def test_noalloc_error_word_is_read_and_cleared():
    """The probe waits on a barrier that nothing completes (2 ms limit): its
    timeout lands in the static scratch, tila_noalloc_read_error returns it,
    and the next tila_launch_noalloc launch starts from a cleared word."""
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    opts = native.default_options(extra=["-DTILA_WAIT_NS=2000000ull"])
    probe = native.Library(native.compile_cubin(PROBE, "tila_noalloc_wait_probe", opts)) \
        .kernel("tila_noalloc_wait_probe")
    status = probe.launch_noalloc((1, 1, 1), (32, 1, 1), [ctypes.c_uint64(0)], 0,
                                  native.ERROR_BLOCK_BYTES, stream=stream)
    assert status == native.TILA_OK, probe.last_log
    word = native.noalloc_read_error(stream, reset=False)
    assert word >> 24 == 1 and word & 0xFFFFFF == 777
    assert native.noalloc_read_error(stream, reset=False) == word      # kept until cleared
    x, reference, rec = _softmax_record(dev, 64, 43)
    assert _noalloc(rec, list(rec.args), native.ERROR_BLOCK_BYTES, stream) == native.TILA_OK
    assert native.noalloc_read_error(stream) == 0                      # the launch cleared it
    tila_b200.check_device_errors(dev)                                 # the normal block is untouched


def test_noalloc_rejects_scratch_beyond_its_capacity():
    dev = torch.device("cuda", 0)
    x, reference, rec = _softmax_record(dev, 8, 42)
    status = _noalloc(rec, list(rec.args), native.NOALLOC_SCRATCH_BYTES + 1, 0)
    assert status == native.TILA_ERR_ARGUMENT
    assert "at most" in rec.entry.kernel.last_log
