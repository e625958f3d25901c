// On-device batch flatten: the per-step bookkeeping of ModelRunner.execute
// (vllmlite/runner.py:66-90) and gather_slots (vllmlite/attention.py:40-44).
//
// One CTA of 1024 threads: the work is a few thousand integer ops, so a single
// CTA (no grid sync, no second launch) has the lowest latency.

#include "batch_meta_kernels.cuh"
#include "meta.cuh"

namespace vllt {

using namespace bmk;

int build_batch_meta(const int32_t* rec, const MetaLayout& L, int bs, int num_blocks, int qp,
                     int32_t* meta, cudaStream_t st, int32_t* pool, int pool_slots, const int32_t* token_src,
                     int token_src_len, int vocab) {
  VLLT_REQUIRE(rec && meta, "build_batch_meta: null pointer");
  VLLT_REQUIRE(bs > 0 && num_blocks > 0 && qp > 0 && vocab > 0, "build_batch_meta: bad sizes");
  VLLT_REQUIRE(!pool || pool_slots > 0, "build_batch_meta: a table pool needs at least one slot");
  VLLT_REQUIRE(!token_src || token_src_len > 0, "build_batch_meta: a token source needs at least one entry");
  VLLT_LAUNCH(1, kThreads, 0, st, build_meta_kernel)(rec, L, bs, num_blocks, qp, meta, pool, pool ? pool_slots : 0,
                                            token_src, token_src ? token_src_len : 0, vocab);
  return check_launch("build_batch_meta");
}

}  // namespace vllt
