// Device code of the KV-cache writes and copy-on-write block copies
// (launched by cache_ops.cu). Plain CUDA C++, so the CPU tests can also run
// it on the host (tests/simt_host.h).
#pragma once

#include <stdint.h>

#include "device_common.cuh"

namespace vllt {
namespace ck {

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

}  // namespace ck
}  // namespace vllt
