// KV-cache writes and copy-on-write block copies.
//
// Cache layout per layer: [num_blocks][n_kv][block_size][head_dim]. A sequence
// position p maps to block table[p / bs], offset p % bs (vllmlite/block.py:154-156);
// the reference's flat "slot" is block * bs + offset.

#include "cache_kernels.cuh"
#include "common.cuh"

namespace vllt {

using namespace ck;

int reshape_and_cache(const void* k, const void* v, void* kc, void* vc, const int32_t* slots,
                      int num_tokens, int n_kv, int D, int bs, int num_blocks, int dtype,
                      cudaStream_t st) {
  if (num_tokens == 0) return VLLT_OK;
  const int esize = dtype == VLLT_F32 ? 4 : 2;
  VLLT_REQUIRE((D * esize) % 16 == 0, "reshape_and_cache: head_dim*elem_size must be a multiple of 16 (D=%d)", D);
  const int64_t vecs = (int64_t)num_tokens * n_kv * (D * esize / 16);
  const int threads = 256;
  const int blocks = (int)std::min<int64_t>((vecs + threads - 1) / threads, 148 * 16);
  const int64_t nslots = (int64_t)num_blocks * bs;
  if (dtype == VLLT_F32)
    VLLT_LAUNCH(blocks, threads, 0, st, reshape_and_cache_kernel<float>)(
        (const float*)k, (const float*)v, (float*)kc, (float*)vc, slots, num_tokens, n_kv, D, bs, nslots);
  else
    VLLT_LAUNCH(blocks, threads, 0, st, reshape_and_cache_kernel<__nv_bfloat16>)(
        (const __nv_bfloat16*)k, (const __nv_bfloat16*)v, (__nv_bfloat16*)kc, (__nv_bfloat16*)vc,
        slots, num_tokens, n_kv, D, bs, nslots);
  return check_launch("reshape_and_cache");
}

int copy_blocks(void* kc, void* vc, const int32_t* pairs, int n_pairs, int n_layers,
                int num_blocks, int n_kv, int bs, int D, int dtype, cudaStream_t st) {
  if (n_pairs == 0) return VLLT_OK;
  const int esize = dtype == VLLT_F32 ? 4 : 2;
  const int64_t block_bytes = (int64_t)n_kv * bs * D * esize;
  VLLT_REQUIRE(block_bytes % 16 == 0, "copy_blocks: block bytes must be a multiple of 16");
  dim3 grid(n_pairs, n_layers, 2);
  VLLT_LAUNCH(grid, 256, 0, st, copy_blocks_kernel)((uint4*)kc, (uint4*)vc, pairs, num_blocks, block_bytes / 16);
  return check_launch("copy_blocks");
}

}  // namespace vllt
