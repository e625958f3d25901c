// Test harness: the library's SIMT kernels compiled for the host and run on
// the fiber emulation of tests/simt_host.h. Each extern "C" entry launches
// one kernel over host buffers with the grid its launcher in the library
// uses; it returns 0, or -1 if the CTA's threads waited on barriers that
// could never complete. Built by the CPU tests with g++ (tests/host_build.py).
#include "simt_host.h"

#include <algorithm>

#include "attention_kernels.cuh"
#include "batch_meta_kernels.cuh"
#include "cache_kernels.cuh"
#include "gemm_f32_kernels.cuh"
#include "norm_kernels.cuh"
#include "sampling_kernels.cuh"

using namespace vllt;

// 0: the default schedule; otherwise the seed of the schedule variation.
extern "C" void set_schedule_seed(uint64_t seed) { simt::schedule_seed() = seed; }

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

// ---- generic paged attention (as attention_pass's generic branch, standalone) ----
// Items are (sequence, tile) pairs from num_seqs and max_qlen; a single-query
// pass over more than 512 keys splits the context when `ws` holds the
// partials (split_len 512), then merges. Returns -1 on a barrier error, -2 for
// a head_dim the library does not build.
namespace {

template <typename T, int D, int ROWS>
bool launch_rows(const ak::AttnParams& p, int items, int splits) {
  return simt::launch(ak::attention_kernel<T, D, ROWS>, dim3(p.n_kv, items, splits), dim3(ak::kWarps * 32),
                      ak::attention_smem_bytes<T, D, ROWS>(), p);
}

template <typename T, int D>
int launch_dim(const ak::AttnParams& p, int rows, int items, int splits) {
  bool ok;
  if (rows <= 2) ok = launch_rows<T, D, 2>(p, items, splits);
  else if (rows <= 4) ok = launch_rows<T, D, 4>(p, items, splits);
  else if (rows <= 8) ok = launch_rows<T, D, 8>(p, items, splits);
  else ok = launch_rows<T, D, 16>(p, items, splits);
  if (!ok) return -1;
  if (splits == 1) return 0;
  const int blocks = (items * p.H * 32 + 255) / 256;
  return simt::launch(ak::merge_splits_kernel<T, D>, dim3(blocks), dim3(256), 0, p, splits) ? 0 : -1;
}

template <typename T>
int launch_any(const ak::AttnParams& p, int D, int rows, int items, int splits) {
  switch (D) {
    case 8: return launch_dim<T, 8>(p, rows, items, splits);
    case 16: return launch_dim<T, 16>(p, rows, items, splits);
    case 32: return launch_dim<T, 32>(p, rows, items, splits);
    case 48: return launch_dim<T, 48>(p, rows, items, splits);
    case 64: return launch_dim<T, 64>(p, rows, items, splits);
    case 128: return launch_dim<T, 128>(p, rows, items, splits);
    default: return -2;
  }
}

}  // namespace

extern "C" int run_attention(int f32, const void* q, const void* kc, const void* vc, void* out, const int32_t* tables,
                             int W, const int32_t* cu_q, const int32_t* ctx, int num_seqs, int max_qlen,
                             int single_query, int max_ctx, int H, int n_kv, int D, int bs, int num_blocks,
                             float scale, float* ws, int64_t ws_bytes) {
  ak::AttnParams p{};
  p.q = q; p.kc = kc; p.vc = vc; p.out = out;
  p.tables = tables; p.W = W; p.cu_q = cu_q; p.ctx = ctx;
  p.H = H; p.n_kv = n_kv; p.n_rep = H / n_kv; p.bs = bs; p.num_blocks = num_blocks;
  p.scale = scale; p.P_cap = num_seqs; p.num_seqs = num_seqs;
  p.qp = single_query ? 1 : vllt::tile_positions(p.n_rep);
  p.items_per_seq = single_query ? 1 : (std::max(max_qlen, 1) + p.qp - 1) / p.qp;
  const int items = p.items_per_seq * num_seqs;
  const int rows = p.qp * p.n_rep;
  int splits = 1;
  if (single_query && max_ctx > 512) {
    splits = (max_ctx + 511) / 512;
    const int64_t need = (int64_t)splits * num_seqs * H * (D + 2) * (int64_t)sizeof(float);
    if (ws && ws_bytes >= need) {
      p.split_len = 512;
      p.ws_o = ws;
      p.ws_ml = ws + (int64_t)splits * num_seqs * H * D;
    } else {
      splits = 1;
    }
  }
  return f32 ? launch_any<float>(p, D, rows, items, splits) : launch_any<__nv_bfloat16>(p, D, rows, items, splits);
}

// ---- fp32 SIMT GEMM (tiles and split-K slices as sgemm_launch / sgemm_go) -------
namespace {

template <int BM, int BN, int BK, int TM, int TN, int THREADS, class Epi>
int sgemm_go_host(const float* A, int lda, const float* B, int ldb, int M_cap, const int* M_dev, int N, int K,
                  const Epi& epi, const GemmScratch* sc) {
  const int k_slice = gemm_k_slice(M_cap, N, K, BM, BN, BK, sc);
  const int ks = ceil_div(K, k_slice);
  return simt::launch(sgemm_kernel<BM, BN, BK, TM, TN, THREADS, Epi>,
                      dim3(ceil_div(N, BN), ceil_div(M_cap, BM), ks), dim3(THREADS), 0, A, lda, B, ldb, M_cap, M_dev,
                      N, K, k_slice, ks > 1 ? sc->partials : nullptr, ks > 1 ? sc->counters : nullptr, epi) ? 0 : -1;
}

template <class Epi>
int sgemm_host(const float* A, int lda, const float* B, int ldb, int M_cap, const int* M_dev, int N, int K,
               const Epi& epi, float* partials, int* counters, int64_t partial_floats, int n_counters) {
  GemmScratch scratch{partials, counters, partial_floats, n_counters};
  const GemmScratch* sc = partials ? &scratch : nullptr;
  if (M_cap <= 16) return sgemm_go_host<16, 64, 32, 2, 4, 128>(A, lda, B, ldb, M_cap, M_dev, N, K, epi, sc);
  if (M_cap <= 32) return sgemm_go_host<32, 64, 32, 4, 4, 128>(A, lda, B, ldb, M_cap, M_dev, N, K, epi, sc);
  if (M_cap <= 64) return sgemm_go_host<64, 64, 16, 4, 4, 256>(A, lda, B, ldb, M_cap, M_dev, N, K, epi, sc);
  return sgemm_go_host<128, 64, 16, 8, 4, 256>(A, lda, B, ldb, M_cap, M_dev, N, K, epi, sc);
}

}  // namespace

#define VLLT_GEMM_ARGS                                                                                           \
  const float *A, int lda, const float *B, int ldb, int M_cap, const int *M_dev, int N, int K, float *partials, \
      int *counters, int64_t partial_floats, int n_counters
#define VLLT_GEMM_PASS A, lda, B, ldb, M_cap, M_dev, N, K

extern "C" int run_sgemm_store(VLLT_GEMM_ARGS, float* C, int ldc, int n_valid) {
  return sgemm_host(VLLT_GEMM_PASS, EpiStore{C, ldc, n_valid}, partials, counters, partial_floats, n_counters);
}

extern "C" int run_sgemm_residual(VLLT_GEMM_ARGS, float* C, int ldc) {
  return sgemm_host(VLLT_GEMM_PASS, EpiResidual{C, ldc}, partials, counters, partial_floats, n_counters);
}

extern "C" int run_sgemm_swiglu(VLLT_GEMM_ARGS, float* out, int ldo) {
  return sgemm_host(VLLT_GEMM_PASS, EpiSwiGLU{out, ldo}, partials, counters, partial_floats, n_counters);
}

extern "C" int run_sgemm_qkv(VLLT_GEMM_ARGS, float* q_out, float* kc, float* vc, const int32_t* pos,
                             const int32_t* slot, const float* cos_t, const float* sin_t, int H, int n_kv, int D,
                             int bs, int max_pos, int64_t num_slots) {
  EpiQKV e{q_out, kc, vc, pos, slot, cos_t, sin_t, H, n_kv, D, bs, max_pos, num_slots};
  return sgemm_host(VLLT_GEMM_PASS, e, partials, counters, partial_floats, n_counters);
}
