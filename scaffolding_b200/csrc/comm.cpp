// Collectives over NCCL (NVLink 5 / NVSwitch), one communicator per
// process/GPU.
//
// The reference has no collective library at all (distributed/__init__.py:19-65
// are no-ops; DataParallel gathers through host NumPy, nn/parallel.py:229-267).
// This file provides the output all-gather of the M-sharded path and a small
// fp32 all-reduce for timing/validation.
//
// NCCL is resolved at run time with dlopen("libnccl.so.2"): if the process
// already has an NCCL loaded (e.g. by a framework) that copy is reused, and
// the engine library itself loads without NCCL present.  Only the handful of
// stable entry points below are used.
#include <dlfcn.h>

#include <mutex>

#include "common.h"

namespace {

// Minimal ABI of the NCCL entry points used (stable since NCCL 2.x).
typedef struct {
  char internal[128];
} NcclUniqueId;
typedef void* NcclComm;
typedef int NcclResult;  // 0 = success, 7 = in progress
enum { kNcclUint8 = 1, kNcclFloat32 = 7 };
enum { kNcclSum = 0, kNcclMax = 2 };

struct NcclApi {
  NcclResult (*get_unique_id)(NcclUniqueId*) = nullptr;
  NcclResult (*comm_init_rank)(NcclComm*, int, NcclUniqueId, int) = nullptr;
  NcclResult (*all_gather)(const void*, void*, size_t, int, NcclComm, cudaStream_t) = nullptr;
  NcclResult (*all_reduce)(const void*, void*, size_t, int, int, NcclComm, cudaStream_t) = nullptr;
  NcclResult (*comm_destroy)(NcclComm) = nullptr;
  NcclResult (*comm_abort)(NcclComm) = nullptr;
  NcclResult (*get_async_error)(NcclComm, NcclResult*) = nullptr;
  NcclResult (*comm_split)(NcclComm, int, int, NcclComm*, void*) = nullptr;
  const char* (*error_string)(NcclResult) = nullptr;
  bool ok = false;
  std::string why;
};

NcclApi& api() {
  static NcclApi a;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) {
      a.why = dlerror() ? dlerror() : "libnccl.so.2 not found";
      return;
    }
#define SF_SYM(field, name)                                                 \
  a.field = reinterpret_cast<decltype(a.field)>(dlsym(h, name));            \
  if (!a.field) {                                                           \
    a.why = std::string("NCCL symbol missing: ") + name;                    \
    return;                                                                 \
  }
    SF_SYM(get_unique_id, "ncclGetUniqueId");
    SF_SYM(comm_init_rank, "ncclCommInitRank");
    SF_SYM(all_gather, "ncclAllGather");
    SF_SYM(all_reduce, "ncclAllReduce");
    SF_SYM(comm_destroy, "ncclCommDestroy");
    SF_SYM(comm_abort, "ncclCommAbort");
    SF_SYM(get_async_error, "ncclCommGetAsyncError");
    SF_SYM(error_string, "ncclGetErrorString");
    SF_SYM(comm_split, "ncclCommSplit");
#undef SF_SYM
    a.ok = true;
  });
  return a;
}

int32_t nccl_fail(NcclResult r, const char* what) {
  NcclApi& a = api();
  return sf::fail(SF_ERR_NCCL, "%s failed: NCCL error %d (%s)", what, r,
                  a.error_string ? a.error_string(r) : "?");
}

#define SF_NCCL_READY()                                                         \
  do {                                                                          \
    if (!api().ok) return sf::fail(SF_ERR_NCCL, "NCCL unavailable: %s", api().why.c_str()); \
  } while (0)

}  // namespace

extern "C" {

int32_t sf_comm_unique_id(uint8_t id_out[128]) {
  if (!id_out) return sf::fail(SF_ERR_INVALID_ARGUMENT, "null output");
  SF_NCCL_READY();
  NcclUniqueId id;
  NcclResult r = api().get_unique_id(&id);
  if (r != 0) return nccl_fail(r, "ncclGetUniqueId");
  memcpy(id_out, id.internal, 128);
  return SF_OK;
}

int32_t sf_comm_init(void** comm, int32_t nranks, int32_t rank, const uint8_t id[128]) {
  if (!comm || !id) return sf::fail(SF_ERR_INVALID_ARGUMENT, "null argument");
  if (nranks < 1 || rank < 0 || rank >= nranks)
    return sf::fail(SF_ERR_INVALID_ARGUMENT, "rank %d / nranks %d", rank, nranks);
  SF_NCCL_READY();
  NcclUniqueId uid;
  memcpy(uid.internal, id, 128);
  NcclComm c = nullptr;
  NcclResult r = api().comm_init_rank(&c, nranks, uid, rank);
  if (r != 0) return nccl_fail(r, "ncclCommInitRank");
  *comm = c;
  return SF_OK;
}

int32_t sf_comm_split(void* comm, int32_t color, int32_t key, void** out) {
  if (!comm || !out) return sf::fail(SF_ERR_INVALID_ARGUMENT, "null argument");
  SF_NCCL_READY();
  NcclComm c = nullptr;
  NcclResult r = api().comm_split(comm, color, key, &c, nullptr);
  if (r != 0) return nccl_fail(r, "ncclCommSplit");
  *out = c;
  return SF_OK;
}

int32_t sf_comm_allgather(void* comm, const void* send, void* recv, size_t bytes_per_rank,
                          void* stream) {
  if (!comm) return sf::fail(SF_ERR_INVALID_ARGUMENT, "null communicator");
  SF_NCCL_READY();
  NcclResult r = api().all_gather(send, recv, bytes_per_rank, kNcclUint8, comm,
                                  static_cast<cudaStream_t>(stream));
  if (r != 0) return nccl_fail(r, "ncclAllGather");
  return SF_OK;
}

int32_t sf_comm_allreduce_f32(void* comm, float* buf, size_t count, int32_t op_max, void* stream) {
  if (!comm) return sf::fail(SF_ERR_INVALID_ARGUMENT, "null communicator");
  SF_NCCL_READY();
  NcclResult r = api().all_reduce(buf, buf, count, kNcclFloat32, op_max ? kNcclMax : kNcclSum, comm,
                                  static_cast<cudaStream_t>(stream));
  if (r != 0) return nccl_fail(r, "ncclAllReduce");
  return SF_OK;
}

int32_t sf_comm_async_error(void* comm, int32_t* nccl_result) {
  if (!comm || !nccl_result) return sf::fail(SF_ERR_INVALID_ARGUMENT, "null argument");
  SF_NCCL_READY();
  NcclResult res = 0;
  NcclResult r = api().get_async_error(comm, &res);
  if (r != 0) return nccl_fail(r, "ncclCommGetAsyncError");
  *nccl_result = res;
  return SF_OK;
}

int32_t sf_comm_abort(void* comm) {
  if (!comm) return SF_OK;
  SF_NCCL_READY();
  NcclResult r = api().comm_abort(comm);
  if (r != 0) return nccl_fail(r, "ncclCommAbort");
  return SF_OK;
}

int32_t sf_comm_destroy(void* comm) {
  if (!comm) return SF_OK;
  SF_NCCL_READY();
  NcclResult r = api().comm_destroy(comm);
  if (r != 0) return nccl_fail(r, "ncclCommDestroy");
  return SF_OK;
}

}  // extern "C"
