// Launch entry point for callers that cannot allocate device memory.
//
// Every kernel this backend generates takes one device word of scratch: the
// error word where bounded waits report a timeout.  The normal entry point
// (tila_launch) expects the caller to pass that word, which the Python host
// allocates once per device.  Some callers cannot do that allocation: code
// that runs while a CUDA graph is being captured (cudaMalloc is not a
// capturable operation), hosts that hand every byte of device memory to
// their own pool and forbid the CUDA allocator, and latency-critical loops
// where cudaMalloc's implicit synchronisation is unacceptable.
// tila_launch_noalloc serves them: the scratch lives in the file-scope array
// below, which every GPU that loads this library holds until the process
// exits.  The entry point itself calls no allocating routine.

#include "../../include/tila_b200.h"

#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <mutex>

namespace {

// Shared scratch for every tila_launch_noalloc call on a device.  Calls that
// overlap on the GPU (different streams, or concurrent host threads) share it
// and therefore race on its contents.
static __device__ __align__(256) unsigned char g_noalloc_scratch[TILA_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
void *g_scratch_ptr[kMaxDevices] = {nullptr};
std::mutex g_setup_mutex;

void put_log(char *log, size_t cap, const char *msg) {
  if (log == nullptr || cap == 0) return;
  std::snprintf(log, cap, "%s", msg);
}

}  // namespace

extern "C" int tila_launch_noalloc(void *kernel, const tila_launch_config *cfg,
                                   void **args, int scratch_arg,
                                   uint32_t scratch_bytes, char *log,
                                   size_t log_cap) {
  if (kernel == nullptr || cfg == nullptr || args == nullptr || scratch_arg < 0)
    return TILA_ERR_ARGUMENT;
  if (scratch_bytes == 0 || scratch_bytes > TILA_NOALLOC_SCRATCH_BYTES) {
    char buf[160];
    std::snprintf(buf, sizeof(buf),
                  "tila_launch_noalloc: kernel needs %u scratch bytes; the static "
                  "scratch holds at most %d",
                  scratch_bytes, TILA_NOALLOC_SCRATCH_BYTES);
    put_log(log, log_cap, buf);
    return TILA_ERR_ARGUMENT;
  }
  int device = -1;
  if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= kMaxDevices) {
    put_log(log, log_cap, "tila_launch_noalloc: no current CUDA device");
    return TILA_ERR_NO_CONTEXT;
  }
  void *scratch = nullptr;
  {
    // One-time set-up per device, with that device current: the address of
    // the array on this device.  In host code g_noalloc_scratch names a host
    // shadow, never a device address, so it is looked up here.
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    if (g_scratch_ptr[device] == nullptr) {
      void *ptr = nullptr;
      cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
      if (e != cudaSuccess || ptr == nullptr) {
        char buf[200];
        std::snprintf(buf, sizeof(buf), "tila_launch_noalloc: cudaGetSymbolAddress failed: %s",
                      cudaGetErrorString(e));
        put_log(log, log_cap, buf);
        return TILA_ERR_DRIVER;
      }
      g_scratch_ptr[device] = ptr;
    }
    scratch = g_scratch_ptr[device];
  }
  // The scratch keeps the previous call's contents: the error word must
  // start at zero, so clear the bytes this launch uses (stream-ordered).
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(static_cast<uintptr_t>(cfg->stream));
  if (cudaMemsetAsync(scratch, 0, scratch_bytes, stream) != cudaSuccess) {
    put_log(log, log_cap, "tila_launch_noalloc: clearing the scratch failed");
    return TILA_ERR_DRIVER;
  }
  void *saved = args[scratch_arg];
  args[scratch_arg] = &scratch;
  int status = tila_launch(kernel, cfg, args, log, log_cap);
  args[scratch_arg] = saved;
  return status;
}
