// Tensor parallelism across GPUs for the decode step (Megatron split).
//
// Each rank holds the rows of q/k/v for its own heads (and so its own KV cache
// columns), the rows of gate/up for its slice of the FFN, and the matching
// input columns of o and down.  The only cross-GPU step is then an all-reduce
// of the o and down projections' partial sums, run with NCCL on the decode
// stream; RMSNorm, the residual, the LM head and the argmax are replicated.
// The reference runs on one device and has no counterpart.
//
// NCCL is reached through dlopen: a process that already loaded libnccl.so.2
// (PyTorch does) shares that copy, so two NCCL builds never meet in one
// process and the library keeps no link-time dependency on NCCL.
#include <dlfcn.h>
#include <nccl.h>

#include <mutex>

#include "common.cuh"

namespace glacier {

namespace {

struct NcclApi {
  decltype(&ncclGetUniqueId) get_unique_id = nullptr;
  decltype(&ncclCommInitRank) comm_init_rank = nullptr;
  decltype(&ncclAllReduce) all_reduce = nullptr;
  decltype(&ncclCommDestroy) comm_destroy = nullptr;
  decltype(&ncclGetErrorString) error_string = nullptr;
  bool ok = false;
};

const NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
    if (!h) return;
    api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
    api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
    api.all_reduce = reinterpret_cast<decltype(api.all_reduce)>(dlsym(h, "ncclAllReduce"));
    api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
    api.error_string = reinterpret_cast<decltype(api.error_string)>(dlsym(h, "ncclGetErrorString"));
    api.ok = api.get_unique_id && api.comm_init_rank && api.all_reduce && api.comm_destroy && api.error_string;
  });
  return api;
}

#define GLC_CHECK_NCCL(expr)                                                                      \
  do {                                                                                            \
    ncclResult_t _r = (expr);                                                                     \
    if (_r != ncclSuccess)                                                                        \
      return ::glacier::set_error(GLACIER_CUDA_ECUDA, "%s failed: %s", #expr, nccl().error_string(_r)); \
  } while (0)

}  // namespace

static_assert(sizeof(ncclUniqueId) == GLACIER_CUDA_TP_ID_BYTES, "NCCL unique id size");

int tp_unique_id(void* out) {
  GLC_REQUIRE(out, "tp_unique_id: null output");
  GLC_REQUIRE(nccl().ok, "tp_unique_id: libnccl.so.2 could not be loaded");
  ncclUniqueId id;
  GLC_CHECK_NCCL(nccl().get_unique_id(&id));
  memcpy(out, &id, sizeof(id));
  return GLACIER_CUDA_OK;
}

int tp_comm_create(void** comm, int rank, int world, const void* id_bytes) {
  GLC_REQUIRE(comm && id_bytes && world >= 2 && rank >= 0 && rank < world, "tp_init: rank %d of %d", rank, world);
  GLC_REQUIRE(nccl().ok, "tp_init: libnccl.so.2 could not be loaded");
  ncclUniqueId id;
  memcpy(&id, id_bytes, sizeof(id));
  ncclComm_t c = nullptr;
  GLC_CHECK_NCCL(nccl().comm_init_rank(&c, world, id, rank));
  *comm = c;
  return GLACIER_CUDA_OK;
}

void tp_comm_destroy(void* comm) {
  if (comm && nccl().ok) nccl().comm_destroy(static_cast<ncclComm_t>(comm));
}

// In-place sum over the ranks of `count` floats on `stream`.
int tp_all_reduce(void* comm, float* buf, size_t count, cudaStream_t stream) {
  GLC_CHECK_NCCL(nccl().all_reduce(buf, buf, count, ncclFloat32, ncclSum, static_cast<ncclComm_t>(comm), stream));
  return GLACIER_CUDA_OK;
}

}  // namespace glacier
