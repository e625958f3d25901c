// Test harness: the library's SIMT kernels compiled for the host and run on
// the fiber emulation of tests/simt_host.h. Each extern "C" entry launches
// one kernel over host buffers with the grid its launcher in the library
// uses; it returns 0, or -1 if the CTA's threads waited on barriers that
// could never complete. Built by the CPU tests with g++ (tests/host_build.py).
#include "simt_host.h"

#include <algorithm>

#include "batch_meta_kernels.cuh"
#include "cache_kernels.cuh"
#include "norm_kernels.cuh"
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

// ---- row-wise kernels (grids as norm.cu's launchers) ---------------------------
static int grid_stride_blocks(int64_t work) { return (int)std::min<int64_t>((work + 255) / 256, 148 * 8); }

extern "C" int run_rmsnorm(const float* x, const int32_t* idx, const float* w, float* out, int rows_cap,
                           const int32_t* rows_dev, int dim, float eps) {
  return simt::launch(nk::rmsnorm_kernel, dim3((rows_cap * 32 + 255) / 256), dim3(256), 0, x, idx, w, out, rows_cap,
                      rows_dev, dim, eps) ? 0 : -1;
}

extern "C" int run_embed(const float* emb, const int32_t* tok, float* x, int T_cap, const int32_t* T_dev, int dim,
                         int vocab) {
  return simt::launch(nk::embed_kernel, dim3(grid_stride_blocks((int64_t)T_cap * dim / 4)), dim3(256), 0, emb, tok,
                      x, T_cap, T_dev, dim, vocab) ? 0 : -1;
}

extern "C" int run_rope(float* x, const int32_t* positions, const float* cos_t, const float* sin_t, int T, int heads,
                        int D, int max_pos) {
  return simt::launch(nk::rope_kernel, dim3(grid_stride_blocks((int64_t)T * heads * (D / 2))), dim3(256), 0, x,
                      positions, cos_t, sin_t, T, heads, D, max_pos) ? 0 : -1;
}

extern "C" int run_embed_bf16(const void* emb, const int32_t* tok, float* x, int T_cap, const int32_t* T_dev,
                              int dim, int vocab) {
  return simt::launch(nk::embed_bf16_kernel, dim3(grid_stride_blocks((int64_t)T_cap * dim / 8)), dim3(256), 0,
                      (const __nv_bfloat16*)emb, tok, x, T_cap, T_dev, dim, vocab) ? 0 : -1;
}

extern "C" int run_rmsnorm_bf16(float* x, const void* add, const int32_t* idx, const float* w, void* out,
                                int rows_cap, const int32_t* rows_dev, int dim, float eps) {
  return simt::launch(nk::rmsnorm_bf16_kernel, dim3(rows_cap), dim3(256), 0, x, (const __nv_bfloat16*)add, idx, w,
                      (__nv_bfloat16*)out, rows_cap, rows_dev, dim, eps) ? 0 : -1;
}

extern "C" int run_argmax_rows(const float* logits, int rows_cap, const int32_t* rows_dev, int vocab, int ld,
                               int offset, float* val, int32_t* idx) {
  return simt::launch(nk::argmax_rows_kernel, dim3(rows_cap), dim3(256), 0, logits, vocab, ld, offset, rows_cap,
                      rows_dev, val, idx) ? 0 : -1;
}

// ---- cache kernels (grids as cache_ops.cu's launchers) -------------------------
extern "C" int run_reshape_and_cache(const void* k, const void* v, void* kc, void* vc, const int32_t* slots,
                                     int num_tokens, int n_kv, int D, int bs, int num_blocks, int f32) {
  const int esize = f32 ? 4 : 2;
  const int64_t vecs = (int64_t)num_tokens * n_kv * (D * esize / 16);
  const dim3 grid((unsigned)std::min<int64_t>((vecs + 255) / 256, 148 * 16));
  const int64_t nslots = (int64_t)num_blocks * bs;
  if (f32)
    return simt::launch(ck::reshape_and_cache_kernel<float>, grid, dim3(256), 0, (const float*)k, (const float*)v,
                        (float*)kc, (float*)vc, slots, num_tokens, n_kv, D, bs, nslots) ? 0 : -1;
  return simt::launch(ck::reshape_and_cache_kernel<__nv_bfloat16>, grid, dim3(256), 0, (const __nv_bfloat16*)k,
                      (const __nv_bfloat16*)v, (__nv_bfloat16*)kc, (__nv_bfloat16*)vc, slots, num_tokens, n_kv, D, bs,
                      nslots) ? 0 : -1;
}

extern "C" int run_copy_blocks(void* kc, void* vc, const int32_t* pairs, int n_pairs, int n_layers, int num_blocks,
                               int n_kv, int bs, int D, int f32) {
  const int64_t block_bytes = (int64_t)n_kv * bs * D * (f32 ? 4 : 2);
  return simt::launch(ck::copy_blocks_kernel, dim3(n_pairs, n_layers, 2), dim3(256), 0, (uint4*)kc, (uint4*)vc,
                      pairs, num_blocks, block_bytes / 16) ? 0 : -1;
}
