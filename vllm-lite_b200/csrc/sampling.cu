// Device sampling: greedy argmax with the reference's pre-steps, speculative
// accept/reject, and temperature / top-k / top-p sampling with the same
// pre-steps and a given uniform.

#include "common.cuh"
#include "sampling_kernels.cuh"

namespace vllt {

using namespace smp;

int sample_greedy(const float* logits, int rows_cap, const int32_t* rows_dev, int vocab, int ld,
                  const uint8_t* eos_mask, int eos_id, const float* penalty, const uint32_t* seen,
                  int32_t* out, cudaStream_t st) {
  if (rows_cap <= 0) return VLLT_OK;
  VLLT_REQUIRE(vocab > 0 && ld >= vocab, "sample_greedy: bad vocab/ld");
  VLLT_LAUNCH(rows_cap, kThreads, 0, st, greedy_kernel)(logits, vocab, ld, eos_mask, eos_id, penalty, seen,
                                               (vocab + 31) / 32, rows_cap, rows_dev, out);
  return check_launch("sample_greedy");
}

int spec_accept(const int32_t* cu_rows, const int32_t* drafts, const int32_t* draft_off,
                int num_seqs, const int32_t* picks, int32_t* n_accepted, cudaStream_t st) {
  if (num_seqs <= 0) return VLLT_OK;
  VLLT_LAUNCH(ceil_div(num_seqs, 128), 128, 0, st, accept_kernel)(cu_rows, drafts, draft_off, num_seqs, picks, n_accepted);
  return check_launch("spec_accept");
}

int sample_top_p(const float* logits, int rows, int vocab, int ld, int logit_rows, const int32_t* row_index,
                 const uint8_t* eos_mask, int eos_id, const float* penalty, const uint32_t* seen,
                 const float* temperature, const int32_t* top_k, const float* top_p, const double* u,
                 int32_t* out, cudaStream_t st) {
  if (rows <= 0) return VLLT_OK;
  VLLT_REQUIRE(vocab > 0 && ld >= vocab && logit_rows > 0 && temperature && u, "sample_top_p: bad arguments");
  VLLT_LAUNCH(rows, kThreads, 0, st, top_p_kernel)(logits, vocab, ld, logit_rows, row_index, eos_mask, eos_id, penalty,
                                          seen, (vocab + 31) / 32, temperature, top_k, top_p, u, out);
  return check_launch("sample_top_p");
}

}  // namespace vllt
