// Multi-GPU gather behind the C ABI (include/tila_b200.h, "multi-GPU"):
// NCCL is opened with dlopen, so the library loads on machines without it;
// when PyTorch already loaded its NCCL, dlopen returns that same copy.

#include "../../include/tila_b200.h"

#include <dlfcn.h>

#include <cstring>
#include <mutex>
#include <string>

namespace {

void put_log(char *log, size_t cap, const std::string &msg) {
  if (log == nullptr || cap == 0) return;
  size_t n = msg.size() < cap - 1 ? msg.size() : cap - 1;
  std::memcpy(log, msg.data(), n);
  log[n] = '\0';
}

// The parts of NCCL's public C API used here (nccl.h): an opaque
// communicator, a 128-byte unique id, int status codes, ncclInt8 = 0.
struct NcclId {
  char internal[TILA_MG_UNIQUE_ID_BYTES];
};
typedef int nccl_result;
typedef void *nccl_comm;

struct Nccl {
  void *handle = nullptr;
  nccl_result (*GetUniqueId)(NcclId *) = nullptr;
  nccl_result (*CommInitRank)(nccl_comm *, int, NcclId, int) = nullptr;
  nccl_result (*AllGather)(const void *, void *, size_t, int, nccl_comm, void *) = nullptr;
  nccl_result (*CommDestroy)(nccl_comm) = nullptr;
  const char *(*GetErrorString)(nccl_result) = nullptr;
  std::string failure;
};

Nccl g_nccl;
std::once_flag g_nccl_once;

template <typename F>
bool bind(void *h, const char *name, F &fn) {
  fn = reinterpret_cast<F>(dlsym(h, name));
  return fn != nullptr;
}

void open_nccl() {
  void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
  if (h == nullptr) {
    const char *e = dlerror();
    g_nccl.failure = std::string("cannot open libnccl.so.2: ") + (e ? e : "?");
    return;
  }
  bool ok = bind(h, "ncclGetUniqueId", g_nccl.GetUniqueId) &&
            bind(h, "ncclCommInitRank", g_nccl.CommInitRank) &&
            bind(h, "ncclAllGather", g_nccl.AllGather) &&
            bind(h, "ncclCommDestroy", g_nccl.CommDestroy) &&
            bind(h, "ncclGetErrorString", g_nccl.GetErrorString);
  if (!ok) {
    g_nccl.failure = "libnccl.so.2 lacks a required entry point";
    return;
  }
  g_nccl.handle = h;
}

int ensure_nccl(char *log, size_t cap) {
  std::call_once(g_nccl_once, open_nccl);
  if (g_nccl.handle == nullptr) {
    put_log(log, cap, g_nccl.failure);
    return TILA_ERR_DRIVER_MISSING;
  }
  return TILA_OK;
}

int check(nccl_result r, const char *what, char *log, size_t cap) {
  if (r == 0) return TILA_OK;
  const char *s = g_nccl.GetErrorString ? g_nccl.GetErrorString(r) : "?";
  put_log(log, cap, std::string(what) + ": " + (s ? s : "?"));
  return TILA_ERR_DRIVER;
}

}  // namespace

extern "C" {

int tila_mg_unique_id(unsigned char id_out[TILA_MG_UNIQUE_ID_BYTES], char *log, size_t log_cap) {
  if (id_out == nullptr) return TILA_ERR_ARGUMENT;
  int st = ensure_nccl(log, log_cap);
  if (st != TILA_OK) return st;
  NcclId id;
  st = check(g_nccl.GetUniqueId(&id), "ncclGetUniqueId", log, log_cap);
  if (st == TILA_OK) std::memcpy(id_out, id.internal, sizeof(id.internal));
  return st;
}

int tila_mg_comm_init(const unsigned char id[TILA_MG_UNIQUE_ID_BYTES], int nranks, int rank,
                      void **comm_out, char *log, size_t log_cap) {
  if (id == nullptr || comm_out == nullptr || nranks < 1 || rank < 0 || rank >= nranks) {
    put_log(log, log_cap, "invalid communicator arguments");
    return TILA_ERR_ARGUMENT;
  }
  int st = ensure_nccl(log, log_cap);
  if (st != TILA_OK) return st;
  NcclId nid;
  std::memcpy(nid.internal, id, sizeof(nid.internal));
  nccl_comm comm = nullptr;
  st = check(g_nccl.CommInitRank(&comm, nranks, nid, rank), "ncclCommInitRank", log, log_cap);
  if (st == TILA_OK) *comm_out = comm;
  return st;
}

int tila_mg_gather(void *comm, const void *sendbuf, void *recvbuf, size_t bytes_per_rank,
                   uint64_t stream, char *log, size_t log_cap) {
  if (comm == nullptr || sendbuf == nullptr || recvbuf == nullptr) {
    put_log(log, log_cap, "null communicator or buffer");
    return TILA_ERR_ARGUMENT;
  }
  int st = ensure_nccl(log, log_cap);
  if (st != TILA_OK) return st;
  return check(g_nccl.AllGather(sendbuf, recvbuf, bytes_per_rank, /*ncclInt8*/ 0, comm,
                                reinterpret_cast<void *>(stream)),
               "ncclAllGather", log, log_cap);
}

int tila_mg_comm_destroy(void *comm) {
  if (comm == nullptr) return TILA_ERR_ARGUMENT;
  if (ensure_nccl(nullptr, 0) != TILA_OK) return TILA_ERR_DRIVER_MISSING;
  return g_nccl.CommDestroy(comm) == 0 ? TILA_OK : TILA_ERR_DRIVER;
}

}  // extern "C"
