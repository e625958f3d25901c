// Device code of the sampling kernels (launched by sampling.cu): greedy
// argmax with the reference's pre-steps, speculative accept, and the
// temperature sampler over sampler_row.cuh. Plain CUDA C++ with no inline
// PTX, so the CPU tests can also run it on the host (tests/simt_host.h).
#pragma once

#include <float.h>
#include <math.h>
#include <stdint.h>

#include "device_common.cuh"
#include "sampler_row.cuh"

namespace vllt {
namespace smp {

constexpr int kThreads = 256;

// (value, index) argmax with the FIRST index winning ties (np.argmax).
struct ArgMax {
  float v;
  int i;
};
__device__ __forceinline__ ArgMax better(ArgMax a, ArgMax b) {
  if (b.v > a.v || (b.v == a.v && b.i < a.i)) return b;
  return a;
}
__device__ ArgMax block_argmax(ArgMax a) {
  __shared__ ArgMax red[kThreads / 32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    ArgMax b{__shfl_xor_sync(0xffffffffu, a.v, o), __shfl_xor_sync(0xffffffffu, a.i, o)};
    a = better(a, b);
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) red[warp] = a;
  __syncthreads();
  if (warp == 0) {
    a = lane < kThreads / 32 ? red[lane] : ArgMax{-INFINITY, INT32_MAX};
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      ArgMax b{__shfl_xor_sync(0xffffffffu, a.v, o), __shfl_xor_sync(0xffffffffu, a.i, o)};
      a = better(a, b);
    }
    if (lane == 0) red[0] = a;
  }
  __syncthreads();
  a = red[0];
  __syncthreads();
  return a;
}

template <typename T, typename Op>
__device__ T block_reduce(T v, Op op, T init) {
  __shared__ T red[kThreads / 32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = op(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    v = lane < kThreads / 32 ? red[lane] : init;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = op(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (lane == 0) red[0] = v;
  }
  __syncthreads();
  v = red[0];
  __syncthreads();
  return v;
}

// sampling.py:41-57, greedy branch: EOS mask (min_tokens), repetition penalty,
// argmax. One CTA per row.
__global__ void greedy_kernel(const float* __restrict__ logits, int vocab, int ld,
                              const uint8_t* __restrict__ eos_mask, int eos_id,
                              const float* __restrict__ penalty, const uint32_t* __restrict__ seen,
                              int seen_words, int rows_cap, const int32_t* rows_dev,
                              int32_t* __restrict__ out) {
  const int rows = rows_dev ? min(*rows_dev, rows_cap) : rows_cap;
  const int r = blockIdx.x;
  if (r >= rows) return;
  const float* x = logits + (int64_t)r * ld;
  const bool mask_eos = eos_mask && eos_mask[r];
  const float pen = penalty ? penalty[r] : 1.0f;
  ArgMax best{-INFINITY, INT32_MAX};
  if (!mask_eos && pen == 1.0f && ((uintptr_t)x & 15) == 0) {  // plain rows: vectorized scan
    row_argmax_part(x, vocab, threadIdx.x, kThreads, best.v, best.i);
  } else {
    for (int c = threadIdx.x; c < vocab; c += kThreads) {
      float v = x[c];
      if (mask_eos && c == eos_id) v = -INFINITY;
      if (pen != 1.0f && seen && ((seen[(int64_t)r * seen_words + (c >> 5)] >> (c & 31)) & 1u))
        v = v > 0.f ? __fdiv_rn(v, pen) : __fmul_rn(v, pen);  // sampling.py:8-13
      best = better(best, ArgMax{v, c});
    }
  }
  best = block_argmax(best);
  if (threadIdx.x == 0) out[r] = best.i == INT32_MAX ? 0 : best.i;
}

// speculative.py:86-100: rows of sequence s are [cu_rows[s], cu_rows[s+1]);
// picks[] already hold each row's argmax. Accept while pick == draft.
__global__ void accept_kernel(const int32_t* __restrict__ cu_rows, const int32_t* __restrict__ drafts,
                              const int32_t* __restrict__ draft_off, int num_seqs,
                              const int32_t* __restrict__ picks, int32_t* __restrict__ n_accepted) {
  const int s = blockIdx.x * blockDim.x + threadIdx.x;
  if (s >= num_seqs) return;
  const int r0 = cu_rows[s], nd = cu_rows[s + 1] - r0 - 1;
  int acc = 0;
  while (acc < nd && picks[r0 + acc] == drafts[draft_off[s] + acc]) ++acc;
  n_accepted[s] = acc;
}

// The CTA of one row as sampler_row.cuh's execution policy: every thread
// takes c = threadIdx.x, + kThreads, ...; reductions are block_reduce; the
// CDF search scans kThreads entries at a time in shared memory (float64),
// carrying the running sum, and stops at the first chunk that holds the
// crossing (the lowest such index wins).
struct BlockPolicy {
  __device__ int tid() const { return threadIdx.x; }
  __device__ int stride() const { return kThreads; }
  __device__ int reduce_sum(int v) { return block_reduce<int>(v, [](int a, int b) { return a + b; }, 0); }
  __device__ float reduce_sum(float v) { return block_reduce<float>(v, [](float a, float b) { return a + b; }, 0.f); }
  __device__ double reduce_sum(double v) {
    return block_reduce<double>(v, [](double a, double b) { return a + b; }, 0.0);
  }
  __device__ float reduce_max(float v) {
    return block_reduce<float>(v, [](float a, float b) { return fmaxf(a, b); }, -INFINITY);
  }
  template <class F>
  __device__ int first_crossing(int n, F pc_of, double u) {
    __shared__ double carry_s;
    __shared__ int pick_s;
    __shared__ double scan[kThreads];
    if (threadIdx.x == 0) {
      carry_s = 0.0;
      pick_s = INT32_MAX;
    }
    __syncthreads();
    for (int base = 0; base < n; base += kThreads) {
      const int c = base + threadIdx.x;
      const double pc = c < n ? pc_of(c) : 0.0;
      scan[threadIdx.x] = pc;  // inclusive scan of pc across the CTA
      __syncthreads();
      for (int o = 1; o < kThreads; o <<= 1) {
        const double add = threadIdx.x >= o ? scan[threadIdx.x - o] : 0.0;
        __syncthreads();
        scan[threadIdx.x] += add;
        __syncthreads();
      }
      const double cdf = carry_s + scan[threadIdx.x];
      const double prev = cdf - pc;
      if (c < n && pc > 0.0 && prev <= u && u < cdf) atomicMin(&pick_s, c);
      __syncthreads();
      if (threadIdx.x == 0) carry_s += scan[kThreads - 1];
      __syncthreads();
      if (pick_s != INT32_MAX) break;  // uniform: every thread reads it after the barrier
    }
    const int pick = pick_s;
    __syncthreads();
    return pick == INT32_MAX ? -1 : pick;
  }
  template <class F>
  __device__ int last(int n, F pred) {
    int best = -1;
    for (int c = threadIdx.x; c < n; c += kThreads)
      if (pred(c)) best = c;
    return block_reduce<int>(best, [](int a, int b) { return a > b ? a : b; }, -1);
  }
};

// The temperature sampler of sampling.py:41-64 (sampler_row.cuh); one CTA per
// row. Row r reads logits row row_index[r] (r when NULL); an index outside
// [0, logit_rows) yields token -1 and nothing else is read.
__global__ void top_p_kernel(const float* __restrict__ logits, int vocab, int ld, int logit_rows,
                             const int32_t* __restrict__ row_index, const uint8_t* __restrict__ eos_mask,
                             int eos_id, const float* __restrict__ penalty, const uint32_t* __restrict__ seen,
                             int seen_words, const float* __restrict__ temperature,
                             const int32_t* __restrict__ top_k, const float* __restrict__ top_p,
                             const double* __restrict__ uni, int32_t* __restrict__ out) {
  const int r = blockIdx.x;
  const int src = row_index ? row_index[r] : r;
  if (src < 0 || src >= logit_rows) {  // uniform across the CTA
    if (threadIdx.x == 0) out[r] = -1;
    return;
  }
  sampler::RowInput row;
  row.x = logits + (int64_t)src * ld;
  row.vocab = vocab;
  row.mask_eos = eos_mask && eos_mask[r] && eos_id >= 0 && eos_id < vocab;
  row.eos_id = eos_id;
  row.pen = penalty ? penalty[r] : 1.f;
  row.seen = (seen && row.pen != 1.f) ? seen + (int64_t)r * seen_words : nullptr;
  row.temp = temperature[r];
  BlockPolicy pol;
  const int pick = sampler::sample_row(pol, row, top_k ? top_k[r] : 0, top_p ? top_p[r] : 1.f, uni[r]);
  if (threadIdx.x == 0) out[r] = pick;
}

}  // namespace smp
}  // namespace vllt
