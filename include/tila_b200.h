/*
 * tila_b200.h - C ABI of the B200 (sm_100a) execution backend for Tila's typed TIR.
 *
 * The reference executes a checked kernel through Triton: runtime.py builds
 * Triton source (lowering.py:136-182), compiles it in backend.preflight
 * (backend.py:61-88) and launches it with `kern[grid](*args, num_warps=...)`
 * (runtime.py:1107).  This library is the native replacement for those three
 * steps.  Python reaches it through ctypes; nothing here takes torch types:
 * device buffers are plain device addresses, streams are CUstream handles cast
 * to uint64_t.
 *
 * Every function returns 0 (TILA_OK) or a negative status code.  The Python
 * host maps the codes onto Tila's diagnostics (TILA-TARGET-010 compile/load,
 * TILA-TARGET-011 resources; backend.py:30-58).  No function aborts the process.
 */
#ifndef TILA_B200_H
#define TILA_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  TILA_OK = 0,
  TILA_ERR_DRIVER_MISSING = -1,  /* libcuda.so.1 could not be opened (no GPU driver) */
  TILA_ERR_DRIVER = -2,          /* a CUDA driver call failed; message in the log buffer */
  TILA_ERR_COMPILE = -3,         /* NVRTC rejected the generated source */
  TILA_ERR_LOAD = -4,            /* the cubin could not be loaded */
  TILA_ERR_RESOURCES = -5,       /* launch exceeds a device limit (smem, threads) */
  TILA_ERR_ARGUMENT = -6,        /* invalid argument to this ABI */
  TILA_ERR_NO_CONTEXT = -7       /* no current CUDA context on the calling thread */
};

/* tila_launch_config.flags */
/* The kernel may be scheduled before the previous kernel in the stream has
 * finished (programmatic dependent launch): its CTAs become resident while the
 * previous grid drains and wait (griddepcontrol.wait) before their first
 * global-memory access.  Every kernel this backend generates performs that
 * wait; kernels from other sources must not be launched with this flag. */
#define TILA_LAUNCH_OVERLAP_PREVIOUS 1u

/* Launch geometry.  grid/block/cluster as in cuLaunchKernelEx; cluster all
 * ones (or zeros) means no cluster.  stream is a CUstream (0 = legacy). */
typedef struct tila_launch_config {
  uint32_t grid[3];
  uint32_t block[3];
  uint32_t cluster[3];
  uint32_t smem_bytes;
  uint64_t stream;
  uint32_t flags;      /* TILA_LAUNCH_* bits */
  uint32_t reserved;   /* must be 0 */
} tila_launch_config;

/* Compiled resource usage of one kernel (backend.py:77-86 reports the same
 * quantities for Triton kernels). */
typedef struct tila_kernel_attrs {
  int32_t registers_per_thread;
  int32_t static_smem_bytes;
  int32_t local_bytes_per_thread; /* > 0 means register spills */
  int32_t max_threads_per_block;
  int32_t max_dynamic_smem_bytes; /* device opt-in limit */
  int32_t binary_version;
} tila_kernel_attrs;

/* Replaces: Triton compile inside backend.preflight (backend.py:65-66).
 * Compiles CUDA C++ source with NVRTC for sm_100a.  On success *cubin_out
 * receives a malloc'ed buffer (release with tila_free_buffer).  The compiler
 * log (warnings or errors) is copied into log (NUL-terminated, truncated to
 * log_cap).  Works without a GPU. */
int tila_nvrtc_compile(const char *source, const char *program_name,
                       const char *const *options, int num_options,
                       void **cubin_out, size_t *cubin_size,
                       char *log, size_t log_cap);

/* NVRTC version, e.g. 12090 for 12.9 (part of the compile cache key). */
int tila_nvrtc_version(int *version_out);

void tila_free_buffer(void *buffer);

/* Loads libcuda.so.1 and calls cuInit.  Idempotent.  Fails with
 * TILA_ERR_DRIVER_MISSING on a machine without the NVIDIA driver. */
int tila_init(char *log, size_t log_cap);

/* Replaces: compiled._init_handles() (backend.py:78).  Loads a cubin as a
 * context-independent CUlibrary, usable on every device of the process. */
int tila_library_load(const void *cubin, size_t size, void **library_out,
                      char *log, size_t log_cap);
int tila_library_unload(void *library);

/* Looks up an extern "C" __global__ function of a loaded library. */
int tila_kernel_get(void *library, const char *name, void **kernel_out,
                    char *log, size_t log_cap);

/* Replaces: the shared-memory / thread checks of backend.preflight
 * (backend.py:71-82).  Reports usage on the current device. */
int tila_kernel_attrs_get(void *kernel, tila_kernel_attrs *out, char *log,
                          size_t log_cap);

/* Replaces: kern[grid](*args, num_warps=...) (runtime.py:1107).  args is the
 * usual cuLaunchKernel parameter array: args[i] points at the value of
 * kernel parameter i.  Raises the kernel's dynamic shared memory limit when
 * cfg->smem_bytes needs it.  Asynchronous on cfg->stream. */
int tila_launch(void *kernel, const tila_launch_config *cfg, void **args,
                char *log, size_t log_cap);

/* Builds a CUtensorMap (128 bytes, 64-byte aligned) for a TMA tile copy.
 * dtype uses CUtensorMapDataType numbering; dims/strides are innermost first,
 * strides in bytes for dims 1..rank-1; box in elements; swizzle uses
 * CUtensorMapSwizzle numbering.  Out-of-bounds elements read as zero. */
int tila_encode_tensor_map(void *tensor_map_out, int dtype, int rank,
                           uint64_t global_address, const uint64_t *dims,
                           const uint64_t *strides_bytes, const uint32_t *box,
                           int swizzle, char *log, size_t log_cap);

/* Capacity of the static scratch used by tila_launch_noalloc. */
#define TILA_NOALLOC_SCRATCH_BYTES 256

/* No counterpart in the reference (its launches allocate through PyTorch).
 * Same as tila_launch, for callers that cannot allocate device memory: hosts
 * whose own pool owns every byte of device memory and forbid the CUDA
 * allocator, and latency-critical loops that cannot afford cudaMalloc's
 * implicit device synchronisation.  args[scratch_arg] (the kernel's scratch
 * pointer: its error block, TILA_ERROR_BLOCK_BYTES) is replaced by the address
 * of a file-scope device array of TILA_NOALLOC_SCRATCH_BYTES bytes, which
 * every GPU that loads this library holds until the process exits; larger
 * scratch_bytes are rejected with TILA_ERR_ARGUMENT.  The first call on a
 * device (and in a new CUDA context) looks up that array's address with the
 * device current, so issue it before any stream capture.  The array is shared
 * by every call and keeps the previous call's contents: its first
 * scratch_bytes are cleared on cfg->stream before the launch, and calls that
 * overlap on the GPU race on it.  Allocates nothing. */
int tila_launch_noalloc(void *kernel, const tila_launch_config *cfg, void **args,
                        int scratch_arg, uint32_t scratch_bytes, char *log,
                        size_t log_cap);

/* No counterpart in the reference.  Reads the error word that the last
 * tila_launch_noalloc launch on the current device recorded in the static
 * scratch ((code << 24) | Tila source line, 0 = none; codes as for the error
 * block below) into *word_out: a 4-byte copy on `stream` after the work
 * already queued there, then a synchronisation of `stream`.  reset != 0
 * clears the word after the copy.  Allocates nothing. */
int tila_noalloc_read_error(uint32_t *word_out, uint64_t stream, int reset,
                            char *log, size_t log_cap);

/* Error block of a launch.  Every generated kernel takes one pointer to a
 * 16-byte device block (the "err" parameter): bytes 0-3 hold the first device
 * error of the launch ((code << 24) | Tila source line; codes: 1 a bounded
 * mbarrier wait timed out, 2 tensor memory allocation failed, 3 a ti.assume
 * was false in a TILA_DEBUG=1 build), bytes 8-15 the device address of a
 * notification word (0 = none).  The thread that records the first error also
 * stores it into the notification word, so a host holding that word in
 * page-locked memory sees device errors without synchronising.  The reference
 * reports device-side failures through Triton's device_assert
 * (lowering.py:339-342); this block is its counterpart. */
#define TILA_ERROR_BLOCK_BYTES 16

/* A zeroed 64-byte page-locked host buffer that kernels can write through
 * *device_address_out (CU_MEMHOSTALLOC_DEVICEMAP | PORTABLE), for the
 * notification word of an error block.  Needs a current context. */
int tila_host_word_alloc(uint32_t **host_out, uint64_t *device_address_out,
                         char *log, size_t log_cap);

/* Frees a buffer from tila_host_word_alloc (no kernel may still write it). */
int tila_host_word_free(uint32_t *host);

/* Number of SMs and opt-in shared memory per block of the current device. */
int tila_device_info(int *sm_count, int *max_smem_optin, int *cc_major,
                     int *cc_minor, char *log, size_t log_cap);

const char *tila_status_string(int status);

/* ---- multi-GPU: gather of output shards (one process per GPU) ----------------
 * The reference has no multi-GPU path; these entry points implement the
 * gather of the grid-partitioned launch (each rank runs a contiguous range of
 * program_id values, then the ranks exchange the rows they wrote) over NCCL,
 * which is opened at run time (libnccl.so.2, the copy PyTorch loaded when it is
 * present).  Communicator handles are opaque; streams are CUstream handles. */
#define TILA_MG_UNIQUE_ID_BYTES 128

/* A fresh communicator id (rank 0 creates it and shares it with the others). */
int tila_mg_unique_id(unsigned char id_out[TILA_MG_UNIQUE_ID_BYTES], char *log,
                      size_t log_cap);

/* Joins the communicator `id` as `rank` of `nranks` on the current device
 * (collective: every rank calls it). */
int tila_mg_comm_init(const unsigned char id[TILA_MG_UNIQUE_ID_BYTES], int nranks,
                      int rank, void **comm_out, char *log, size_t log_cap);

/* recvbuf[r * bytes_per_rank .. (r + 1) * bytes_per_rank) = rank r's sendbuf,
 * for every rank r (an all-gather; every rank calls it, asynchronously on
 * `stream`).  sendbuf may alias this rank's slot of recvbuf. */
int tila_mg_gather(void *comm, const void *sendbuf, void *recvbuf, size_t bytes_per_rank,
                   uint64_t stream, char *log, size_t log_cap);

int tila_mg_comm_destroy(void *comm);

#ifdef __cplusplus
}
#endif

#endif /* TILA_B200_H */
