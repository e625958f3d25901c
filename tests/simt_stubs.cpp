// Test infrastructure: the parts of libvllt the host build leaves out
// (tests/host_build.py build_library_host): the tensor-core prefill attention
// (attention_pass then takes the CUDA-core kernel) and NCCL's all-reduce
// (tensor parallelism). They report themselves unsupported.
#include <cuda_runtime.h>
#include <stdint.h>

#include "../include/vllt.h"
#include "ops.cuh"

namespace vllt {

void set_error(const char* fmt, ...);

int tp_allreduce_bf16(void*, int64_t, void*, cudaStream_t) {
  set_error("tensor-parallel all-reduce: not in the host build (NCCL)");
  return VLLT_ERR_UNSUPPORTED;
}

bool prefill_tc_supported(const AttnCall&) { return false; }
int prefill_tc_positions(int n_rep) { return n_rep >= 16 ? 1 : 16 / n_rep; }
int prefill_tc_pass(const AttnCall&, int, const int32_t*, const int32_t*, const int32_t*, int, int, int, int*,
                    cudaStream_t) {
  set_error("tensor-core prefill: not in the host build");
  return VLLT_ERR_UNSUPPORTED;
}

}  // namespace vllt

// The emulation's schedule for every launch of the host build: 0 is the
// default, any other value seeds the shuffled schedule (tests/simt_host.h).
extern "C" void vllt_host_schedule_seed(uint64_t seed) { simt::schedule_seed() = seed; }
