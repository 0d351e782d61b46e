// Native launcher of the B200 backend: NVRTC compilation, cubin loading,
// kernel launch and TMA descriptor encoding behind the C ABI declared in
// include/tila_b200.h.
//
// The CUDA driver is opened with dlopen so that this library loads (and the
// NVRTC half works) on machines without a GPU driver.  Kernels are loaded as
// CUlibrary objects (CUDA 12 "context-independent loading"), so one load
// serves every device the process touches; launches go to the caller's
// current context, which PyTorch sets for the tensor's device.

#include "../../include/tila_b200.h"

#include <cuda.h>
#include <dlfcn.h>
#include <nvrtc.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

namespace {

void put_log(char *log, size_t cap, const std::string &msg) {
  if (log == nullptr || cap == 0) return;
  size_t n = msg.size() < cap - 1 ? msg.size() : cap - 1;
  std::memcpy(log, msg.data(), n);
  log[n] = '\0';
}

// Driver entry points, resolved once from libcuda.so.1.
struct Driver {
  void *handle = nullptr;
  CUresult (*Init)(unsigned int) = nullptr;
  CUresult (*GetErrorString)(CUresult, const char **) = nullptr;
  CUresult (*CtxGetCurrent)(CUcontext *) = nullptr;
  CUresult (*CtxGetDevice)(CUdevice *) = nullptr;
  CUresult (*DeviceGetAttribute)(int *, CUdevice_attribute, CUdevice) = nullptr;
  CUresult (*LibraryLoadData)(CUlibrary *, const void *, CUjit_option *, void **,
                              unsigned int, CUlibraryOption *, void **,
                              unsigned int) = nullptr;
  CUresult (*LibraryUnload)(CUlibrary) = nullptr;
  CUresult (*LibraryGetKernel)(CUkernel *, CUlibrary, const char *) = nullptr;
  CUresult (*KernelGetAttribute)(int *, CUfunction_attribute, CUkernel,
                                 CUdevice) = nullptr;
  CUresult (*KernelSetAttribute)(CUfunction_attribute, int, CUkernel,
                                 CUdevice) = nullptr;
  CUresult (*LaunchKernelEx)(const CUlaunchConfig *, CUfunction, void **,
                             void **) = nullptr;
  CUresult (*TensorMapEncodeTiled)(CUtensorMap *, CUtensorMapDataType,
                                   cuuint32_t, void *, const cuuint64_t *,
                                   const cuuint64_t *, const cuuint32_t *,
                                   const cuuint32_t *, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion,
                                   CUtensorMapFloatOOBfill) = nullptr;
  CUresult (*MemHostAlloc)(void **, size_t, unsigned int) = nullptr;
  CUresult (*MemHostGetDevicePointer)(CUdeviceptr *, void *, unsigned int) = nullptr;
  CUresult (*MemFreeHost)(void *) = nullptr;
  bool ready = false;
  std::string failure;
};

Driver g_drv;
std::once_flag g_drv_once;

template <typename F>
bool bind(void *h, const char *name, F &fn) {
  fn = reinterpret_cast<F>(dlsym(h, name));
  return fn != nullptr;
}

void open_driver() {
  void *h = dlopen("libcuda.so.1", RTLD_NOW | RTLD_GLOBAL);
  if (h == nullptr) {
    const char *e = dlerror();
    g_drv.failure = std::string("cannot open libcuda.so.1: ") + (e ? e : "?");
    return;
  }
  g_drv.handle = h;
  bool ok = bind(h, "cuInit", g_drv.Init) &&
            bind(h, "cuGetErrorString", g_drv.GetErrorString) &&
            bind(h, "cuCtxGetCurrent", g_drv.CtxGetCurrent) &&
            bind(h, "cuCtxGetDevice", g_drv.CtxGetDevice) &&
            bind(h, "cuDeviceGetAttribute", g_drv.DeviceGetAttribute) &&
            bind(h, "cuLibraryLoadData", g_drv.LibraryLoadData) &&
            bind(h, "cuLibraryUnload", g_drv.LibraryUnload) &&
            bind(h, "cuLibraryGetKernel", g_drv.LibraryGetKernel) &&
            bind(h, "cuKernelGetAttribute", g_drv.KernelGetAttribute) &&
            bind(h, "cuKernelSetAttribute", g_drv.KernelSetAttribute) &&
            bind(h, "cuLaunchKernelEx", g_drv.LaunchKernelEx) &&
            bind(h, "cuTensorMapEncodeTiled", g_drv.TensorMapEncodeTiled) &&
            bind(h, "cuMemHostAlloc", g_drv.MemHostAlloc) &&
            bind(h, "cuMemHostGetDevicePointer_v2", g_drv.MemHostGetDevicePointer) &&
            bind(h, "cuMemFreeHost", g_drv.MemFreeHost);
  if (!ok) {
    g_drv.failure = "libcuda.so.1 lacks a required entry point (driver too old?)";
    return;
  }
  CUresult r = g_drv.Init(0);
  if (r != CUDA_SUCCESS) {
    const char *s = nullptr;
    g_drv.GetErrorString(r, &s);
    g_drv.failure = std::string("cuInit failed: ") + (s ? s : "?");
    return;
  }
  g_drv.ready = true;
}

int ensure_driver(char *log, size_t cap) {
  std::call_once(g_drv_once, open_driver);
  if (!g_drv.ready) {
    put_log(log, cap, g_drv.failure);
    return g_drv.handle == nullptr ? TILA_ERR_DRIVER_MISSING : TILA_ERR_DRIVER;
  }
  return TILA_OK;
}

int driver_error(CUresult r, const char *what, char *log, size_t cap,
                 int code = TILA_ERR_DRIVER) {
  const char *s = nullptr;
  if (g_drv.GetErrorString) g_drv.GetErrorString(r, &s);
  char buf[512];
  std::snprintf(buf, sizeof(buf), "%s failed: %s (CUresult %d)", what,
                s ? s : "unknown error", static_cast<int>(r));
  put_log(log, cap, buf);
  return code;
}

int current_device(CUdevice *dev, char *log, size_t cap) {
  CUcontext ctx = nullptr;
  CUresult r = g_drv.CtxGetCurrent(&ctx);
  if (r != CUDA_SUCCESS) return driver_error(r, "cuCtxGetCurrent", log, cap);
  if (ctx == nullptr) {
    put_log(log, cap, "no current CUDA context (initialise the device first)");
    return TILA_ERR_NO_CONTEXT;
  }
  r = g_drv.CtxGetDevice(dev);
  if (r != CUDA_SUCCESS) return driver_error(r, "cuCtxGetDevice", log, cap);
  return TILA_OK;
}

}  // namespace

// The calling thread's current CUDA context (for the no-allocation entry
// point, which caches a device address per context); not part of the ABI.
int tila_internal_current_context(void **ctx_out) {
  if (ensure_driver(nullptr, 0) != TILA_OK) return TILA_ERR_DRIVER;
  CUcontext ctx = nullptr;
  if (g_drv.CtxGetCurrent(&ctx) != CUDA_SUCCESS) return TILA_ERR_DRIVER;
  *ctx_out = ctx;
  return TILA_OK;
}

extern "C" {

const char *tila_status_string(int status) {
  switch (status) {
    case TILA_OK: return "ok";
    case TILA_ERR_DRIVER_MISSING: return "CUDA driver not available";
    case TILA_ERR_DRIVER: return "CUDA driver call failed";
    case TILA_ERR_COMPILE: return "NVRTC compilation failed";
    case TILA_ERR_LOAD: return "cubin load failed";
    case TILA_ERR_RESOURCES: return "launch exceeds device resources";
    case TILA_ERR_ARGUMENT: return "invalid argument";
    case TILA_ERR_NO_CONTEXT: return "no current CUDA context";
    default: return "unknown status";
  }
}

int tila_nvrtc_version(int *version_out) {
  if (version_out == nullptr) return TILA_ERR_ARGUMENT;
  int major = 0, minor = 0;
  if (nvrtcVersion(&major, &minor) != NVRTC_SUCCESS) return TILA_ERR_COMPILE;
  *version_out = major * 1000 + minor * 10;
  return TILA_OK;
}

int tila_nvrtc_compile(const char *source, const char *program_name,
                       const char *const *options, int num_options,
                       void **cubin_out, size_t *cubin_size, char *log,
                       size_t log_cap) {
  if (source == nullptr || cubin_out == nullptr || cubin_size == nullptr ||
      num_options < 0)
    return TILA_ERR_ARGUMENT;
  *cubin_out = nullptr;
  *cubin_size = 0;
  nvrtcProgram prog;
  nvrtcResult r = nvrtcCreateProgram(&prog, source,
                                     program_name ? program_name : "tila.cu",
                                     0, nullptr, nullptr);
  if (r != NVRTC_SUCCESS) {
    put_log(log, log_cap, std::string("nvrtcCreateProgram: ") + nvrtcGetErrorString(r));
    return TILA_ERR_COMPILE;
  }
  r = nvrtcCompileProgram(prog, num_options, options);
  size_t log_size = 0;
  nvrtcGetProgramLogSize(prog, &log_size);
  std::string text(log_size, '\0');
  if (log_size > 0) nvrtcGetProgramLog(prog, &text[0]);
  while (!text.empty() && text.back() == '\0') text.pop_back();
  put_log(log, log_cap, text);
  if (r != NVRTC_SUCCESS) {
    nvrtcDestroyProgram(&prog);
    return TILA_ERR_COMPILE;
  }
  size_t n = 0;
  if (nvrtcGetCUBINSize(prog, &n) != NVRTC_SUCCESS || n == 0) {
    nvrtcDestroyProgram(&prog);
    put_log(log, log_cap, "NVRTC produced no cubin (is -arch=sm_100a set?)");
    return TILA_ERR_COMPILE;
  }
  void *buf = std::malloc(n);
  if (buf == nullptr) {
    nvrtcDestroyProgram(&prog);
    return TILA_ERR_RESOURCES;
  }
  nvrtcGetCUBIN(prog, static_cast<char *>(buf));
  nvrtcDestroyProgram(&prog);
  *cubin_out = buf;
  *cubin_size = n;
  return TILA_OK;
}

void tila_free_buffer(void *buffer) { std::free(buffer); }

int tila_init(char *log, size_t log_cap) { return ensure_driver(log, log_cap); }

int tila_library_load(const void *cubin, size_t size, void **library_out,
                      char *log, size_t log_cap) {
  if (cubin == nullptr || size == 0 || library_out == nullptr) return TILA_ERR_ARGUMENT;
  int st = ensure_driver(log, log_cap);
  if (st != TILA_OK) return st;
  CUlibrary lib = nullptr;
  CUresult r = g_drv.LibraryLoadData(&lib, cubin, nullptr, nullptr, 0, nullptr,
                                     nullptr, 0);
  if (r != CUDA_SUCCESS) return driver_error(r, "cuLibraryLoadData", log, log_cap, TILA_ERR_LOAD);
  *library_out = lib;
  return TILA_OK;
}

int tila_library_unload(void *library) {
  if (library == nullptr) return TILA_ERR_ARGUMENT;
  int st = ensure_driver(nullptr, 0);
  if (st != TILA_OK) return st;
  return g_drv.LibraryUnload(static_cast<CUlibrary>(library)) == CUDA_SUCCESS
             ? TILA_OK : TILA_ERR_DRIVER;
}

int tila_kernel_get(void *library, const char *name, void **kernel_out,
                    char *log, size_t log_cap) {
  if (library == nullptr || name == nullptr || kernel_out == nullptr) return TILA_ERR_ARGUMENT;
  int st = ensure_driver(log, log_cap);
  if (st != TILA_OK) return st;
  CUkernel k = nullptr;
  CUresult r = g_drv.LibraryGetKernel(&k, static_cast<CUlibrary>(library), name);
  if (r != CUDA_SUCCESS) return driver_error(r, "cuLibraryGetKernel", log, log_cap, TILA_ERR_LOAD);
  *kernel_out = k;
  return TILA_OK;
}

int tila_kernel_attrs_get(void *kernel, tila_kernel_attrs *out, char *log,
                          size_t log_cap) {
  if (kernel == nullptr || out == nullptr) return TILA_ERR_ARGUMENT;
  int st = ensure_driver(log, log_cap);
  if (st != TILA_OK) return st;
  CUdevice dev;
  st = current_device(&dev, log, log_cap);
  if (st != TILA_OK) return st;
  CUkernel k = static_cast<CUkernel>(kernel);
  struct { CUfunction_attribute a; int32_t *dst; } q[] = {
      {CU_FUNC_ATTRIBUTE_NUM_REGS, &out->registers_per_thread},
      {CU_FUNC_ATTRIBUTE_SHARED_SIZE_BYTES, &out->static_smem_bytes},
      {CU_FUNC_ATTRIBUTE_LOCAL_SIZE_BYTES, &out->local_bytes_per_thread},
      {CU_FUNC_ATTRIBUTE_MAX_THREADS_PER_BLOCK, &out->max_threads_per_block},
      {CU_FUNC_ATTRIBUTE_BINARY_VERSION, &out->binary_version},
  };
  for (auto &e : q) {
    int v = 0;
    CUresult r = g_drv.KernelGetAttribute(&v, e.a, k, dev);
    if (r != CUDA_SUCCESS) return driver_error(r, "cuKernelGetAttribute", log, log_cap);
    *e.dst = v;
  }
  int optin = 0;
  CUresult r = g_drv.DeviceGetAttribute(
      &optin, CU_DEVICE_ATTRIBUTE_MAX_SHARED_MEMORY_PER_BLOCK_OPTIN, dev);
  if (r != CUDA_SUCCESS) return driver_error(r, "cuDeviceGetAttribute", log, log_cap);
  out->max_dynamic_smem_bytes = optin - out->static_smem_bytes;
  return TILA_OK;
}

int tila_launch(void *kernel, const tila_launch_config *cfg, void **args,
                char *log, size_t log_cap) {
  if (kernel == nullptr || cfg == nullptr) return TILA_ERR_ARGUMENT;
  for (int i = 0; i < 3; ++i)
    if (cfg->block[i] == 0) return TILA_ERR_ARGUMENT;
  if ((cfg->flags & ~TILA_LAUNCH_OVERLAP_PREVIOUS) != 0 || cfg->reserved != 0) {
    put_log(log, log_cap, "tila_launch: unknown flag bits");
    return TILA_ERR_ARGUMENT;
  }
  int st = ensure_driver(log, log_cap);
  if (st != TILA_OK) return st;
  if (cfg->grid[0] == 0 || cfg->grid[1] == 0 || cfg->grid[2] == 0) return TILA_OK;
  CUdevice dev;
  st = current_device(&dev, log, log_cap);
  if (st != TILA_OK) return st;
  CUkernel k = static_cast<CUkernel>(kernel);
  if (cfg->smem_bytes > 48 * 1024) {
    int optin = 0;
    g_drv.DeviceGetAttribute(&optin, CU_DEVICE_ATTRIBUTE_MAX_SHARED_MEMORY_PER_BLOCK_OPTIN, dev);
    int stat = 0;
    g_drv.KernelGetAttribute(&stat, CU_FUNC_ATTRIBUTE_SHARED_SIZE_BYTES, k, dev);
    if (static_cast<long>(cfg->smem_bytes) + stat > optin) {
      char buf[256];
      std::snprintf(buf, sizeof(buf),
                    "shared memory: required %u dynamic + %d static bytes, limit %d",
                    cfg->smem_bytes, stat, optin);
      put_log(log, log_cap, buf);
      return TILA_ERR_RESOURCES;
    }
    CUresult r = g_drv.KernelSetAttribute(
        CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES,
        static_cast<int>(cfg->smem_bytes), k, dev);
    if (r != CUDA_SUCCESS) return driver_error(r, "cuKernelSetAttribute", log, log_cap, TILA_ERR_RESOURCES);
  }
  CUlaunchConfig lc;
  std::memset(&lc, 0, sizeof(lc));
  lc.gridDimX = cfg->grid[0];
  lc.gridDimY = cfg->grid[1];
  lc.gridDimZ = cfg->grid[2];
  lc.blockDimX = cfg->block[0];
  lc.blockDimY = cfg->block[1];
  lc.blockDimZ = cfg->block[2];
  lc.sharedMemBytes = cfg->smem_bytes;
  lc.hStream = reinterpret_cast<CUstream>(static_cast<uintptr_t>(cfg->stream));
  CUlaunchAttribute attr[2];
  unsigned nattr = 0;
  unsigned cx = cfg->cluster[0] ? cfg->cluster[0] : 1;
  unsigned cy = cfg->cluster[1] ? cfg->cluster[1] : 1;
  unsigned cz = cfg->cluster[2] ? cfg->cluster[2] : 1;
  if (cx * cy * cz > 1) {
    attr[nattr].id = CU_LAUNCH_ATTRIBUTE_CLUSTER_DIMENSION;
    attr[nattr].value.clusterDim.x = cx;
    attr[nattr].value.clusterDim.y = cy;
    attr[nattr].value.clusterDim.z = cz;
    ++nattr;
  }
  if (cfg->flags & TILA_LAUNCH_OVERLAP_PREVIOUS) {
    attr[nattr].id = CU_LAUNCH_ATTRIBUTE_PROGRAMMATIC_STREAM_SERIALIZATION;
    attr[nattr].value.programmaticStreamSerializationAllowed = 1;
    ++nattr;
  }
  lc.attrs = nattr ? attr : nullptr;
  lc.numAttrs = nattr;
  // A CUkernel is accepted wherever a CUfunction is expected; the driver
  // resolves it for the current context.
  CUresult r = g_drv.LaunchKernelEx(&lc, reinterpret_cast<CUfunction>(k), args, nullptr);
  if (r != CUDA_SUCCESS) {
    int code = (r == CUDA_ERROR_OUT_OF_MEMORY || r == CUDA_ERROR_LAUNCH_OUT_OF_RESOURCES ||
                r == CUDA_ERROR_INVALID_VALUE)
                   ? TILA_ERR_RESOURCES : TILA_ERR_DRIVER;
    return driver_error(r, "cuLaunchKernelEx", log, log_cap, code);
  }
  return TILA_OK;
}

int tila_encode_tensor_map(void *tensor_map_out, int dtype, int rank,
                           uint64_t global_address, const uint64_t *dims,
                           const uint64_t *strides_bytes, const uint32_t *box,
                           int swizzle, char *log, size_t log_cap) {
  if (tensor_map_out == nullptr || rank < 1 || rank > 5 || dims == nullptr ||
      box == nullptr || (rank > 1 && strides_bytes == nullptr))
    return TILA_ERR_ARGUMENT;
  if ((reinterpret_cast<uintptr_t>(tensor_map_out) & 63u) != 0) {
    put_log(log, log_cap, "tensor map storage must be 64-byte aligned");
    return TILA_ERR_ARGUMENT;
  }
  int st = ensure_driver(log, log_cap);
  if (st != TILA_OK) return st;
  cuuint32_t elem_strides[5] = {1, 1, 1, 1, 1};
  CUresult r = g_drv.TensorMapEncodeTiled(
      static_cast<CUtensorMap *>(tensor_map_out),
      static_cast<CUtensorMapDataType>(dtype), static_cast<cuuint32_t>(rank),
      reinterpret_cast<void *>(static_cast<uintptr_t>(global_address)),
      reinterpret_cast<const cuuint64_t *>(dims),
      reinterpret_cast<const cuuint64_t *>(strides_bytes),
      reinterpret_cast<const cuuint32_t *>(box), elem_strides,
      CU_TENSOR_MAP_INTERLEAVE_NONE, static_cast<CUtensorMapSwizzle>(swizzle),
      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return driver_error(r, "cuTensorMapEncodeTiled", log, log_cap, TILA_ERR_ARGUMENT);
  return TILA_OK;
}

int tila_host_word_alloc(uint32_t **host_out, uint64_t *device_address_out,
                         char *log, size_t log_cap) {
  if (host_out == nullptr || device_address_out == nullptr) return TILA_ERR_ARGUMENT;
  int st = ensure_driver(log, log_cap);
  if (st != TILA_OK) return st;
  CUdevice dev;
  st = current_device(&dev, log, log_cap);
  if (st != TILA_OK) return st;
  void *p = nullptr;
  CUresult r = g_drv.MemHostAlloc(&p, 64, CU_MEMHOSTALLOC_PORTABLE | CU_MEMHOSTALLOC_DEVICEMAP);
  if (r != CUDA_SUCCESS) return driver_error(r, "cuMemHostAlloc", log, log_cap);
  std::memset(p, 0, 64);
  CUdeviceptr d = 0;
  r = g_drv.MemHostGetDevicePointer(&d, p, 0);
  if (r != CUDA_SUCCESS) {
    g_drv.MemFreeHost(p);
    return driver_error(r, "cuMemHostGetDevicePointer", log, log_cap);
  }
  *host_out = static_cast<uint32_t *>(p);
  *device_address_out = static_cast<uint64_t>(d);
  return TILA_OK;
}

int tila_host_word_free(uint32_t *host) {
  if (host == nullptr) return TILA_OK;
  if (ensure_driver(nullptr, 0) != TILA_OK) return TILA_ERR_DRIVER;
  return g_drv.MemFreeHost(host) == CUDA_SUCCESS ? TILA_OK : TILA_ERR_DRIVER;
}

int tila_device_info(int *sm_count, int *max_smem_optin, int *cc_major,
                     int *cc_minor, char *log, size_t log_cap) {
  int st = ensure_driver(log, log_cap);
  if (st != TILA_OK) return st;
  CUdevice dev;
  st = current_device(&dev, log, log_cap);
  if (st != TILA_OK) return st;
  struct { CUdevice_attribute a; int *dst; } q[] = {
      {CU_DEVICE_ATTRIBUTE_MULTIPROCESSOR_COUNT, sm_count},
      {CU_DEVICE_ATTRIBUTE_MAX_SHARED_MEMORY_PER_BLOCK_OPTIN, max_smem_optin},
      {CU_DEVICE_ATTRIBUTE_COMPUTE_CAPABILITY_MAJOR, cc_major},
      {CU_DEVICE_ATTRIBUTE_COMPUTE_CAPABILITY_MINOR, cc_minor},
  };
  for (auto &e : q) {
    if (e.dst == nullptr) continue;
    CUresult r = g_drv.DeviceGetAttribute(e.dst, e.a, dev);
    if (r != CUDA_SUCCESS) return driver_error(r, "cuDeviceGetAttribute", log, log_cap);
  }
  return TILA_OK;
}

}  // extern "C"
