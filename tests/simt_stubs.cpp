// Test infrastructure: the tensor-core paths of libvllt (bf16 forward,
// tensor-core prefill attention) for the host build (tests/host_build.py
// build_library_host). They report themselves unsupported; the fp32 forward
// and the CUDA-core attention kernels never select them.
#include <cuda_runtime.h>
#include <stdint.h>

#include "../include/vllt.h"
#include "ops.cuh"

namespace vllt {

void set_error(const char* fmt, ...);

int forward_bf16(const vllt_model_desc*, const int32_t*, const vllt_caps*, const vllt_step_bounds*, void*, void*,
                 int64_t, float*, cudaStream_t) {
  set_error("bf16 forward: not in the host build");
  return VLLT_ERR_UNSUPPORTED;
}
int64_t forward_bf16_ws_bytes(const vllt_model_desc*, const vllt_caps*) { return 0; }

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
