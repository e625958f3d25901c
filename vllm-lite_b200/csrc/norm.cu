// Row-wise layer pieces: RMSNorm (optionally gathering rows), token embedding,
// standalone RoPE.

#include "common.cuh"
#include "norm_kernels.cuh"

namespace vllt {

using namespace nk;

int embed_bf16(const void* emb, const int32_t* tok, float* x, int T_cap, const int32_t* T_dev, int dim,
               int vocab, cudaStream_t st) {
  if (T_cap <= 0) return VLLT_OK;
  VLLT_REQUIRE(dim % 8 == 0, "embed_bf16: dim must be a multiple of 8");
  const int64_t vecs = (int64_t)T_cap * dim / 8;
  const int blocks = (int)std::min<int64_t>((vecs + 255) / 256, 148 * 8);
  VLLT_LAUNCH(blocks, 256, 0, st, embed_bf16_kernel)((const __nv_bfloat16*)emb, tok, x, T_cap, T_dev, dim, vocab);
  return check_launch("embed_bf16");
}

int rmsnorm_bf16(float* x, const void* add, const int32_t* idx, const float* w, void* out, int rows_cap,
                 const int32_t* rows_dev, int dim, float eps, cudaStream_t st) {
  if (rows_cap <= 0) return VLLT_OK;
  VLLT_REQUIRE(dim % 4 == 0, "rmsnorm_bf16: dim must be a multiple of 4");
  VLLT_LAUNCH(rows_cap, 256, 0, st, rmsnorm_bf16_kernel)(x, (const __nv_bfloat16*)add, idx, w, (__nv_bfloat16*)out, rows_cap,
                                                rows_dev, dim, eps);
  return check_launch("rmsnorm_bf16");
}

int argmax_rows(const float* logits, int rows_cap, const int32_t* rows_dev, int vocab, int ld, int offset,
                float* val, int32_t* idx, cudaStream_t st) {
  if (rows_cap <= 0) return VLLT_OK;
  VLLT_LAUNCH(rows_cap, 256, 0, st, argmax_rows_kernel)(logits, vocab, ld, offset, rows_cap, rows_dev, val, idx);
  return check_launch("argmax_rows");
}

int rmsnorm(const float* x, const int32_t* idx, const float* w, float* out, int rows_cap,
            const int32_t* rows_dev, int dim, float eps, cudaStream_t st) {
  if (rows_cap <= 0) return VLLT_OK;
  VLLT_REQUIRE(dim % 4 == 0, "rmsnorm: dim must be a multiple of 4");
  const int threads = 256;
  const int blocks = ceil_div(rows_cap * 32, threads);
  VLLT_LAUNCH(blocks, threads, 0, st, rmsnorm_kernel)(x, idx, w, out, rows_cap, rows_dev, dim, eps);
  return check_launch("rmsnorm");
}

int embed(const float* emb, const int32_t* tok, float* x, int T_cap, const int32_t* T_dev, int dim,
          int vocab, cudaStream_t st) {
  if (T_cap <= 0) return VLLT_OK;
  VLLT_REQUIRE(dim % 4 == 0, "embed: dim must be a multiple of 4");
  const int64_t vecs = (int64_t)T_cap * dim / 4;
  const int blocks = (int)std::min<int64_t>((vecs + 255) / 256, 148 * 8);
  VLLT_LAUNCH(blocks, 256, 0, st, embed_kernel)(emb, tok, x, T_cap, T_dev, dim, vocab);
  return check_launch("embed");
}

int rope(float* x, const int32_t* positions, const float* cos_t, const float* sin_t, int T,
         int heads, int D, int max_pos, cudaStream_t st) {
  if (T <= 0) return VLLT_OK;
  VLLT_REQUIRE(D % 2 == 0, "rope: head_dim must be even");
  const int64_t total = (int64_t)T * heads * (D / 2);
  const int blocks = (int)std::min<int64_t>((total + 255) / 256, 148 * 8);
  VLLT_LAUNCH(blocks, 256, 0, st, rope_kernel)(x, positions, cos_t, sin_t, T, heads, D, max_pos);
  return check_launch("rope");
}

}  // namespace vllt
