// Test harness: the library's SIMT kernels compiled for the host and run on
// the fiber emulation of tests/simt_host.h. Each extern "C" entry launches
// one kernel over host buffers with the grid its launcher in the library
// uses; it returns 0, or -1 if the CTA's threads waited on barriers that
// could never complete. Built by the CPU tests with g++ (tests/host_build.py).
#include "simt_host.h"

#include "batch_meta_kernels.cuh"
#include "sampling_kernels.cuh"

using namespace vllt;

extern "C" int run_greedy(const float* logits, int rows, int vocab, int ld, const uint8_t* eos_mask, int eos_id,
                          const float* penalty, const uint32_t* seen, const int32_t* rows_dev, int32_t* out) {
  return simt::launch(smp::greedy_kernel, dim3(rows), dim3(smp::kThreads), 0, logits, vocab, ld, eos_mask, eos_id,
                      penalty, seen, (vocab + 31) / 32, rows, rows_dev, out) ? 0 : -1;
}

extern "C" int run_top_p(const float* logits, int rows, int vocab, int ld, int logit_rows, const int32_t* row_index,
                         const uint8_t* eos_mask, int eos_id, const float* penalty, const uint32_t* seen,
                         const float* temperature, const int32_t* top_k, const float* top_p, const double* u,
                         int32_t* out) {
  return simt::launch(smp::top_p_kernel, dim3(rows), dim3(smp::kThreads), 0, logits, vocab, ld, logit_rows,
                      row_index, eos_mask, eos_id, penalty, seen, (vocab + 31) / 32, temperature, top_k, top_p, u,
                      out) ? 0 : -1;
}

extern "C" int run_accept(const int32_t* cu_rows, const int32_t* drafts, const int32_t* draft_off, int num_seqs,
                          const int32_t* picks, int32_t* n_accepted) {
  return simt::launch(smp::accept_kernel, dim3((num_seqs + 127) / 128), dim3(128), 0, cu_rows, drafts, draft_off,
                      num_seqs, picks, n_accepted) ? 0 : -1;
}

extern "C" int run_build_meta(const int32_t* rec, int32_t* pool, int pool_slots, int S_cap, int T_cap, int R_cap,
                              int W_cap, int bs, int num_blocks, int qp, int32_t* meta, const int32_t* tsrc,
                              int tsrc_len, int vocab) {
  const MetaLayout L = MetaLayout::make(S_cap, T_cap, R_cap, W_cap);
  return simt::launch(bmk::build_meta_kernel, dim3(1), dim3(bmk::kThreads), 0, rec, L, bs, num_blocks, qp, meta,
                      pool, pool ? pool_slots : 0, tsrc, tsrc ? tsrc_len : 0, vocab) ? 0 : -1;
}
