// Test infrastructure: the part of libvllt the host build leaves out
// (tests/host_build.py build_library_host): NCCL's all-reduce (tensor
// parallelism), which becomes a call of a host collective that a test
// registers (vllt_host_set_allreduce) and otherwise reports itself
// unsupported; and the test hooks of the emulation.
#include <cuda_runtime.h>
#include <stdint.h>

#include "../include/vllt.h"
#include "ops.cuh"
#include "simt_tc.h"

namespace vllt {

void set_error(const char* fmt, ...);

// In-place sum over the ranks of `count` bf16 values at buf (ncclAllReduce,
// ncclBfloat16, ncclSum on the GPU); 0 on success.
typedef int (*HostAllReduce)(void* buf, int64_t count, void* comm);
static HostAllReduce g_host_allreduce = nullptr;

// The forward's call site is the GPU build's (forward_bf16.cu); the launches
// before it have completed on the emulation, so the buffer holds this rank's
// partial when the collective runs.
int tp_allreduce_bf16(void* buf, int64_t count, void* comm, cudaStream_t) {
  if (count <= 0) return VLLT_OK;
  VLLT_REQUIRE(comm, "tp_allreduce: no communicator");
  if (!g_host_allreduce) {
    set_error("tensor-parallel all-reduce: not in the host build (NCCL) and no host collective registered");
    return VLLT_ERR_UNSUPPORTED;
  }
  if (g_host_allreduce(buf, count, comm) != 0) {
    set_error("tensor-parallel all-reduce: the host collective failed");
    return VLLT_ERR_CUDA;
  }
  return VLLT_OK;
}

}  // namespace vllt

// Register (or, with null, remove) the host collective the forward's
// all-reduce calls.
extern "C" void vllt_host_set_allreduce(vllt::HostAllReduce f) { vllt::g_host_allreduce = f; }

// The emulation's schedule for every launch of the host build: 0 is the
// default, any other value seeds the shuffled schedule (tests/simt_host.h).
extern "C" void vllt_host_schedule_seed(uint64_t seed) { simt::schedule_seed() = seed; }
// Drop the n-th tensor-map load of the tensor-core kernels from now on
// (1: the next one; 0: none): its bytes never arrive, so a bounded wait expires.
extern "C" void vllt_host_drop_tma(int64_t n) { simt::tensor::drop_countdown() = n; }
// tcgen05.mma instructions the emulation has executed so far.
extern "C" int64_t vllt_host_mma_count() { return simt::tensor::mma_count().load(); }
