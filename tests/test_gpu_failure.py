"""Failure detection on the GPU without a GPU fault.

Every wait of a generated kernel (an mbarrier that a TMA copy, an MMA commit
or the partner warpgroup completes) is bounded: after TILA_WAIT_NS it records
"mbarrier wait timed out" and the source line in the launch's error word,
marks the CTA dead so that its later waits return at once, and the kernel
runs to its end.  Here a kernel waits on a barrier that nothing ever
completes, under a 2 ms limit; the host reads the status, and the context
stays usable for the next launch."""

import ctypes

import numpy as np
import pytest

import tila_b200
from tila_b200 import native, workloads as W

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

SOURCE = r'''
#include "tila_tile.cuh"
extern "C" __global__ void tila_wait_timeout_probe(tila::u32 *err, long long *out) {
  __shared__ __align__(8) tila::u64 bar;
  __shared__ int dead;
  if (threadIdx.x == 0) { tila::mbar_init(&bar, 1); dead = 0; tila::mbar_fence_init(); }
  __syncthreads();
  if (threadIdx.x == 0) {
    const long long t0 = (long long)tila::globaltimer_ns();
    const bool ok = tila::mbar_wait(&bar, 0u, err, 4242u, &dead);
    out[0] = ok ? 1 : 0;
    out[1] = (long long)tila::globaltimer_ns() - t0;
  }
  __syncthreads();
  const long long t1 = (long long)tila::globaltimer_ns();
  const bool ok2 = tila::mbar_wait(&bar, 0u, err, 4343u, &dead);
  if (threadIdx.x == 1) {
    out[2] = ok2 ? 1 : 0;
    out[3] = (long long)tila::globaltimer_ns() - t1;
  }
}
'''


def test_bounded_wait_reports_timeout_and_context_survives():
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    opts = native.default_options(extra=["-DTILA_WAIT_NS=2000000ull"])
    lib = native.Library(native.compile_cubin(SOURCE, "tila_wait_timeout_probe", opts))
    kern = lib.kernel("tila_wait_timeout_probe")
    err = torch.zeros(native.ERROR_BLOCK_BYTES // 4, dtype=torch.int32, device=dev)   # no host word
    out = torch.full((4,), -1, dtype=torch.int64, device=dev)
    kern.launch((1, 1, 1), (32, 1, 1), [ctypes.c_void_p(err.data_ptr()), ctypes.c_void_p(out.data_ptr())],
                stream=torch.cuda.current_stream(dev).cuda_stream)
    torch.cuda.synchronize()
    word = int(err[0].item()) & 0xFFFFFFFF
    assert word >> 24 == 1                      # kErrMbarrierTimeout
    assert word & 0xFFFFFF == 4242              # the first wait that gave up
    first_ok, first_ns, second_ok, second_ns = out.tolist()
    assert first_ok == 0 and 2_000_000 <= first_ns < 1_000_000_000
    assert second_ok == 0 and second_ns < 1_000_000   # later waits return at once
    # the context is intact: a generated kernel runs and matches the interpreter
    x, y = W.add_inputs(4096, seed=3)
    o = torch.zeros(4096, device=dev)
    W.add_kernel[(4,)](torch.from_numpy(x).to(dev), torch.from_numpy(y).to(dev), o, BLOCK=1024)
    assert tila_b200.read_device_errors(dev) == 0
    np.testing.assert_array_equal(o.cpu().numpy(), x + y)


def test_device_error_raises_at_the_next_launch():
    """A launch that recorded a device error (here the timed-out wait of the
    probe, given the backend's error block for the device) makes the next
    kernel[grid] call on that device raise TILA-TARGET-005 with the recorded
    line, without the host synchronising; the launch after that runs."""
    from tila_b200.backend import _error_word
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    opts = native.default_options(extra=["-DTILA_WAIT_NS=2000000ull"])
    lib = native.Library(native.compile_cubin(SOURCE, "tila_wait_timeout_probe", opts))
    kern = lib.kernel("tila_wait_timeout_probe")
    x, y = W.add_inputs(4096, seed=4)
    xg, yg = torch.from_numpy(x).to(dev), torch.from_numpy(y).to(dev)
    o = torch.zeros(4096, device=dev)
    W.add_kernel[(4,)](xg, yg, o, BLOCK=1024)              # creates the device's error block
    out = torch.full((4,), -1, dtype=torch.int64, device=dev)
    kern.launch((1, 1, 1), (32, 1, 1), [ctypes.c_void_p(_error_word(dev).data_ptr()),
                                        ctypes.c_void_p(out.data_ptr())],
                stream=torch.cuda.current_stream(dev).cuda_stream)
    torch.cuda.synchronize()
    with pytest.raises(tila_b200.tila.errors.TilaError) as exc:
        W.add_kernel[(4,)](xg, yg, o, BLOCK=1024)
    assert exc.value.code == "TILA-TARGET-005"
    assert exc.value.loc.line == 4242 and "timed out" in str(exc.value)
    o.zero_()
    W.add_kernel[(4,)](xg, yg, o, BLOCK=1024)               # reported once; the device is usable
    torch.cuda.synchronize()
    tila_b200.check_device_errors(dev)
    assert tila_b200.read_device_errors(dev) == 0
    np.testing.assert_array_equal(o.cpu().numpy(), x + y)


def test_debug_assume_stops_the_program_and_raises(tmp_path, monkeypatch):
    """TILA_DEBUG=1: a false ti.assume raises like the interpreter's
    device_assert; the indices stay inside the buffer, so nothing unsafe runs."""
    import semantics_support as S
    monkeypatch.setenv("TILA_DEBUG", "1")
    k = S.assume_gather_program(tmp_path)
    n = 100
    rng = np.random.default_rng(3)
    idx = rng.integers(0, n, size=n).astype(np.int32)
    data = rng.standard_normal(n).astype(np.float32)
    dev = torch.device("cuda", 0)
    gi, gd = torch.from_numpy(idx).to(dev), torch.from_numpy(data).to(dev)
    out = torch.zeros(n, device=dev)
    k[(2,)](gi, gd, out, n)                      # every assumption holds
    torch.cuda.synchronize()
    np.testing.assert_array_equal(out.cpu().numpy(), data[idx])
    with pytest.raises(AssertionError, match="ti.assume"):
        k[(2,)](gi, gd, out, 50)                 # idx < 50 is false for some lanes
    assert tila_b200.read_device_errors(dev) == 0
    out.zero_()
    k[(2,)](gi, gd, out, n)                      # the next launch runs normally
    torch.cuda.synchronize()
    np.testing.assert_array_equal(out.cpu().numpy(), data[idx])
