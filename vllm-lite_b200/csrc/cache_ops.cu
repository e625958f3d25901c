// KV-cache writes and copy-on-write block copies.
//
// Cache layout per layer: [num_blocks][n_kv][block_size][head_dim]. A sequence
// position p maps to block table[p / bs], offset p % bs (vllmlite/block.py:154-156);
// the reference's flat "slot" is block * bs + offset.

#include "common.cuh"

namespace vllt {

// One CTA per group of tokens; each thread moves 16-byte vectors of one
// (token, head) row. Memory bound: 2 * T * n_kv * D * esize bytes read+written.
template <typename T>
__global__ void reshape_and_cache_kernel(const T* __restrict__ k, const T* __restrict__ v,
                                         T* __restrict__ kc, T* __restrict__ vc,
                                         const int32_t* __restrict__ slots, int num_tokens,
                                         int n_kv, int D, int bs, int64_t num_slots) {
  constexpr int VEC = 16 / sizeof(T);
  const int vecs_per_row = D / VEC;
  const int per_token = n_kv * vecs_per_row;
  const int64_t total = (int64_t)num_tokens * per_token;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int t = (int)(i / per_token);
    const int r = (int)(i % per_token);
    const int h = r / vecs_per_row;
    const int c = r % vecs_per_row;
    const int64_t slot = slots[t];
    if (slot < 0 || slot >= num_slots) continue;
    const int64_t blk = slot / bs, off = slot % bs;
    const int64_t src = ((int64_t)t * n_kv + h) * D + (int64_t)c * VEC;
    const int64_t dst = ((blk * n_kv + h) * bs + off) * D + (int64_t)c * VEC;
    *reinterpret_cast<uint4*>(kc + dst) = *reinterpret_cast<const uint4*>(k + src);
    *reinterpret_cast<uint4*>(vc + dst) = *reinterpret_cast<const uint4*>(v + src);
  }
}

// grid = (pairs, layers, 2): K and V of one block of one layer per CTA.
__global__ void copy_blocks_kernel(uint4* __restrict__ kc, uint4* __restrict__ vc,
                                   const int32_t* __restrict__ pairs, int num_blocks,
                                   int64_t block_vecs) {
  const int p = blockIdx.x, layer = blockIdx.y;
  uint4* base = blockIdx.z ? vc : kc;
  const int src = pairs[2 * p], dst = pairs[2 * p + 1];
  if (src < 0 || src >= num_blocks || dst < 0 || dst >= num_blocks) return;
  const int64_t lo = (int64_t)layer * num_blocks * block_vecs;
  const uint4* s = base + lo + (int64_t)src * block_vecs;
  uint4* d = base + lo + (int64_t)dst * block_vecs;
  for (int64_t i = threadIdx.x; i < block_vecs; i += blockDim.x) d[i] = s[i];
}

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
    reshape_and_cache_kernel<float><<<blocks, threads, 0, st>>>(
        (const float*)k, (const float*)v, (float*)kc, (float*)vc, slots, num_tokens, n_kv, D, bs, nslots);
  else
    reshape_and_cache_kernel<__nv_bfloat16><<<blocks, threads, 0, st>>>(
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
  copy_blocks_kernel<<<grid, 256, 0, st>>>((uint4*)kc, (uint4*)vc, pairs, num_blocks, block_bytes / 16);
  return check_launch("copy_blocks");
}

}  // namespace vllt
