// Tensor-parallel communicator: NCCL loaded at run time (dlopen), so the
// library has no link-time NCCL dependency and single-GPU users never load it.
// Used by the bf16 forward for the all-reduce after o_proj and down_proj
// (row-parallel projections) and by the vocab-parallel greedy pick.

#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>

#include "ops.cuh"

namespace vllt {

namespace {

struct NcclApi {
  decltype(&ncclGetUniqueId) get_unique_id = nullptr;
  decltype(&ncclCommInitRank) init_rank = nullptr;
  decltype(&ncclCommDestroy) destroy = nullptr;
  decltype(&ncclAllReduce) all_reduce = nullptr;
  decltype(&ncclAllGather) all_gather = nullptr;
  decltype(&ncclGetErrorString) error_string = nullptr;
  bool ok = false;
};

NcclApi& nccl() {
  static NcclApi api;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
    api.get_unique_id = (decltype(api.get_unique_id))dlsym(h, "ncclGetUniqueId");
    api.init_rank = (decltype(api.init_rank))dlsym(h, "ncclCommInitRank");
    api.destroy = (decltype(api.destroy))dlsym(h, "ncclCommDestroy");
    api.all_reduce = (decltype(api.all_reduce))dlsym(h, "ncclAllReduce");
    api.all_gather = (decltype(api.all_gather))dlsym(h, "ncclAllGather");
    api.error_string = (decltype(api.error_string))dlsym(h, "ncclGetErrorString");
    api.ok = api.get_unique_id && api.init_rank && api.destroy && api.all_reduce && api.all_gather;
  });
  return api;
}

int nccl_status(ncclResult_t r, const char* what) {
  if (r == ncclSuccess) return VLLT_OK;
  set_error("%s: %s", what, nccl().error_string ? nccl().error_string(r) : "nccl error");
  return VLLT_ERR_CUDA;
}

}  // namespace

int tp_allreduce_bf16(void* buf, int64_t count, void* comm, cudaStream_t st) {
  if (count <= 0) return VLLT_OK;
  VLLT_REQUIRE(comm && nccl().ok, "tp_allreduce: no communicator");
  return nccl_status(nccl().all_reduce(buf, buf, (size_t)count, ncclBfloat16, ncclSum, (ncclComm_t)comm, st),
                     "ncclAllReduce");
}

int tp_allgather_bytes(const void* send, void* recv, int64_t bytes, void* comm, cudaStream_t st) {
  VLLT_REQUIRE(comm && nccl().ok, "tp_allgather: no communicator");
  return nccl_status(nccl().all_gather(send, recv, (size_t)bytes, ncclUint8, (ncclComm_t)comm, st),
                     "ncclAllGather");
}

}  // namespace vllt

using namespace vllt;

extern "C" {

int vllt_tp_unique_id(uint8_t* out128) {
  clear_error();
  VLLT_REQUIRE(out128, "tp_unique_id: null output");
  if (!nccl().ok) {
    set_error("tp_unique_id: libnccl.so.2 could not be loaded");
    return VLLT_ERR_UNSUPPORTED;
  }
  ncclUniqueId id;
  const int rc = nccl_status(nccl().get_unique_id(&id), "ncclGetUniqueId");
  if (rc == VLLT_OK) memcpy(out128, id.internal, NCCL_UNIQUE_ID_BYTES);
  return rc;
}

int vllt_tp_init(const uint8_t* id128, int32_t rank, int32_t world, void** comm_out) {
  clear_error();
  VLLT_REQUIRE(id128 && comm_out && world >= 1 && rank >= 0 && rank < world, "tp_init: bad arguments");
  if (!nccl().ok) {
    set_error("tp_init: libnccl.so.2 could not be loaded");
    return VLLT_ERR_UNSUPPORTED;
  }
  ncclUniqueId id;
  memcpy(id.internal, id128, NCCL_UNIQUE_ID_BYTES);
  ncclComm_t comm = nullptr;
  const int rc = nccl_status(nccl().init_rank(&comm, world, id, rank), "ncclCommInitRank");
  *comm_out = rc == VLLT_OK ? (void*)comm : nullptr;
  return rc;
}

int vllt_tp_destroy(void* comm) {
  clear_error();
  if (!comm) return VLLT_OK;
  VLLT_REQUIRE(nccl().ok, "tp_destroy: NCCL not loaded");
  return nccl_status(nccl().destroy((ncclComm_t)comm), "ncclCommDestroy");
}

int vllt_tp_allreduce_bf16(void* buf, int64_t count, void* comm, void* stream) {
  clear_error();
  return tp_allreduce_bf16(buf, count, comm, as_stream(stream));
}

}  // extern "C"
