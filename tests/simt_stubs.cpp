// Test infrastructure: the part of libvllt the host build leaves out
// (tests/host_build.py build_library_host): NCCL's all-reduce (tensor
// parallelism), which reports itself unsupported; and the test hooks of the
// emulation.
#include <cuda_runtime.h>
#include <stdint.h>

#include "../include/vllt.h"
#include "ops.cuh"
#include "simt_tc.h"

namespace vllt {

void set_error(const char* fmt, ...);

int tp_allreduce_bf16(void*, int64_t, void*, cudaStream_t) {
  set_error("tensor-parallel all-reduce: not in the host build (NCCL)");
  return VLLT_ERR_UNSUPPORTED;
}

}  // namespace vllt

// The emulation's schedule for every launch of the host build: 0 is the
// default, any other value seeds the shuffled schedule (tests/simt_host.h).
extern "C" void vllt_host_schedule_seed(uint64_t seed) { simt::schedule_seed() = seed; }
// Drop the n-th tensor-map load of the tensor-core kernels from now on
// (1: the next one; 0: none): its bytes never arrive, so a bounded wait expires.
extern "C" void vllt_host_drop_tma(int64_t n) { simt::tensor::drop_countdown() = n; }
// tcgen05.mma instructions the emulation has executed so far.
extern "C" int64_t vllt_host_mma_count() { return simt::tensor::mma_count().load(); }
