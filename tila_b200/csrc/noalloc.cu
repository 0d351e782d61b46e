// Launch entry point for callers that cannot allocate device memory.
//
// Every kernel this backend generates takes a small scratch block in global
// memory: its error block (TILA_ERROR_BLOCK_BYTES), where bounded waits and
// debug assumptions record the first device error.  The normal entry point
// (tila_launch) expects the caller to pass that block, which the Python host
// allocates once per device.  Some callers cannot make that allocation:
// hosts that hand every byte of device memory to their own pool and forbid
// the CUDA allocator, and latency-critical loops where cudaMalloc's implicit
// device synchronisation is unacceptable.  tila_launch_noalloc serves them:
// the scratch lives in the file-scope array below, which every GPU that loads
// this library holds until the process exits, and tila_noalloc_read_error
// lets them read what a launch recorded there.  Neither entry point calls an
// allocating routine.

#include "../../include/tila_b200.h"

#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <mutex>

// launcher.cpp: the calling thread's current CUDA context.
int tila_internal_current_context(void **ctx_out);

namespace {

// Shared scratch for every tila_launch_noalloc call on a device.  Calls that
// overlap on the GPU (different streams, or concurrent host threads) share it
// and therefore race on its contents.
static __device__ __align__(256) unsigned char g_noalloc_scratch[TILA_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
// The array's device address per device, with the CUDA context it was looked
// up in: a launch under another context (a non-primary context, or the
// primary context after a reset) looks the address up again.
void *g_scratch_ptr[kMaxDevices] = {nullptr};
void *g_scratch_ctx[kMaxDevices] = {nullptr};
std::mutex g_setup_mutex;

void put_log(char *log, size_t cap, const char *msg) {
  if (log == nullptr || cap == 0) return;
  std::snprintf(log, cap, "%s", msg);
}

// The device address of g_noalloc_scratch in the current context, looked up
// once per (device, context) with that device current.  In host code the name
// g_noalloc_scratch denotes a host-side shadow of the array, never a device
// address, so it is never passed to a kernel directly.
int scratch_address(void **out, char *log, size_t log_cap) {
  int device = -1;
  if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= kMaxDevices) {
    put_log(log, log_cap, "tila_launch_noalloc: no current CUDA device");
    return TILA_ERR_NO_CONTEXT;
  }
  void *ctx = nullptr;
  int st = tila_internal_current_context(&ctx);
  if (st != TILA_OK || ctx == nullptr) {
    put_log(log, log_cap, "tila_launch_noalloc: no current CUDA context");
    return TILA_ERR_NO_CONTEXT;
  }
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (g_scratch_ptr[device] == nullptr || g_scratch_ctx[device] != ctx) {
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
    g_scratch_ctx[device] = ctx;
  }
  *out = g_scratch_ptr[device];
  return TILA_OK;
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
  void *scratch = nullptr;
  int status = scratch_address(&scratch, log, log_cap);
  if (status != TILA_OK) return status;
  // The scratch keeps the previous call's contents: the error word must
  // start at zero, so clear the bytes this launch uses (stream-ordered).
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(static_cast<uintptr_t>(cfg->stream));
  if (cudaMemsetAsync(scratch, 0, scratch_bytes, stream) != cudaSuccess) {
    put_log(log, log_cap, "tila_launch_noalloc: clearing the scratch failed");
    return TILA_ERR_DRIVER;
  }
  void *saved = args[scratch_arg];
  args[scratch_arg] = &scratch;
  status = tila_launch(kernel, cfg, args, log, log_cap);
  args[scratch_arg] = saved;
  return status;
}

extern "C" int tila_noalloc_read_error(uint32_t *word_out, uint64_t stream, int reset,
                                       char *log, size_t log_cap) {
  if (word_out == nullptr) return TILA_ERR_ARGUMENT;
  void *scratch = nullptr;
  int status = scratch_address(&scratch, log, log_cap);
  if (status != TILA_OK) return status;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(static_cast<uintptr_t>(stream));
  uint32_t word = 0;
  if (cudaMemcpyAsync(&word, scratch, sizeof(word), cudaMemcpyDeviceToHost, s) != cudaSuccess ||
      (reset && cudaMemsetAsync(scratch, 0, sizeof(word), s) != cudaSuccess) ||
      cudaStreamSynchronize(s) != cudaSuccess) {
    put_log(log, log_cap, "tila_noalloc_read_error: reading the static scratch failed");
    return TILA_ERR_DRIVER;
  }
  *word_out = word;
  return TILA_OK;
}
