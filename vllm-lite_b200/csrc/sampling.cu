// Device sampling: greedy argmax with the reference's pre-steps, speculative
// accept/reject, and temperature / top-k / top-p sampling with the same
// pre-steps and a given uniform.

#include <float.h>
#include <math.h>

#include "common.cuh"

namespace vllt {

namespace {

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

// Map a float to an unsigned key with the same order (for bisection).
__device__ __forceinline__ uint32_t order_key(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// The full sampler of sampling.py:41-64 for temperature rows; one CTA per row.
// The row's logits pass through the reference's pre-steps on the fly, in its
// order: EOS masked to -inf while min_tokens is not reached (:51-52), the
// repetition penalty on every token the row has seen (:54, :8-13), division by
// the temperature (:59); then top-k (:16-20), top-p (:23-33) and the draw
// (:63-64). The k-th largest value and the nucleus threshold are found by
// bisection over order keys, so any vocab size works with O(32 * vocab) work
// and no sort. The draw is numpy's Generator.choice with the uniform `uni[r]`
// it would have taken from the request's generator: the first index whose
// float64 CDF (cumulative sum of the kept probabilities, divided by the total)
// exceeds u. Row r reads logits row row_index[r] (r when NULL); an index
// outside [0, logit_rows) yields token -1 and nothing else is read.
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
  const float* x = logits + (int64_t)src * ld;
  const bool mask_eos = eos_mask && eos_mask[r] && eos_id >= 0 && eos_id < vocab;
  const float pen = penalty ? penalty[r] : 1.f;
  const uint32_t* sb = (seen && pen != 1.f) ? seen + (int64_t)r * seen_words : nullptr;
  const float temp = temperature[r];
  const int k = top_k ? top_k[r] : 0;
  const float p = top_p ? top_p[r] : 1.f;
  auto val = [&](int c) {
    float v = x[c];
    if (mask_eos && c == eos_id) v = -INFINITY;
    if (sb && ((sb[c >> 5] >> (c & 31)) & 1u)) v = v > 0.f ? __fdiv_rn(v, pen) : __fmul_rn(v, pen);
    return __fdiv_rn(v, temp);
  };

  // top-k: the largest key v with count(x >= v) >= k
  uint32_t cut_key = 0;
  if (k > 0 && k < vocab) {
    uint32_t lo = 0, hi = 0xffffffffu;
    while (lo < hi) {
      const uint32_t mid = lo + (hi - lo + 1) / 2;
      int cnt = 0;
      for (int c = threadIdx.x; c < vocab; c += kThreads) cnt += order_key(val(c)) >= mid;
      cnt = block_reduce<int>(cnt, [](int a, int b) { return a + b; }, 0);
      if (cnt >= k) lo = mid; else hi = mid - 1;
    }
    cut_key = lo;
  }
  auto kept_k = [&](float v) { return order_key(v) >= cut_key; };
  float mx = -INFINITY;
  for (int c = threadIdx.x; c < vocab; c += kThreads) {
    const float v = val(c);
    if (kept_k(v)) mx = fmaxf(mx, v);
  }
  mx = block_reduce<float>(mx, [](float a, float b) { return fmaxf(a, b); }, -INFINITY);
  float sum = 0.f;
  for (int c = threadIdx.x; c < vocab; c += kThreads) {
    const float v = val(c);
    if (kept_k(v)) sum += expf(v - mx);
  }
  sum = block_reduce<float>(sum, [](float a, float b) { return a + b; }, 0.f);
  // top-p: smallest probability b with G(b) = sum_{p_j > b} p_j < p; keep p_i >= b
  float pmin = 0.f;
  if (p < 1.f) {
    uint32_t lo = __float_as_uint(0.f), hi = __float_as_uint(1.f);
    while (lo < hi) {
      const uint32_t mid = lo + (hi - lo) / 2;
      const float b = __uint_as_float(mid);
      float g = 0.f;
      for (int c = threadIdx.x; c < vocab; c += kThreads) {
        const float v = val(c);
        if (kept_k(v)) {
          const float pc = __fdiv_rn(expf(v - mx), sum);
          if (pc > b) g += pc;
        }
      }
      g = block_reduce<float>(g, [](float a, float b2) { return a + b2; }, 0.f);
      if (g < p) hi = mid; else lo = mid + 1;
    }
    pmin = __uint_as_float(lo);
  }
  auto kept = [&](float v) {
    return kept_k(v) && (p >= 1.f || __fdiv_rn(expf(v - mx), sum) >= pmin);
  };
  // renormalised probabilities, CDF in vocab order (numpy's choice: cumsum in
  // float64, divided by the total, first index with cdf > u)
  float s2 = 0.f;
  for (int c = threadIdx.x; c < vocab; c += kThreads) {
    const float v = val(c);
    if (kept(v)) s2 += expf(v - mx);
  }
  s2 = block_reduce<float>(s2, [](float a, float b) { return a + b; }, 0.f);
  __shared__ double carry_s;
  __shared__ int pick_s;
  if (threadIdx.x == 0) { carry_s = 0.0; pick_s = -1; }
  __syncthreads();
  double total = 0.0;
  for (int c = threadIdx.x; c < vocab; c += kThreads) {
    const float v = val(c);
    if (kept(v)) total += (double)__fdiv_rn(expf(v - mx), s2);
  }
  total = block_reduce<double>(total, [](double a, double b) { return a + b; }, 0.0);
  const double u = uni[r] * total;
  for (int base = 0; base < vocab; base += kThreads) {
    const int c = base + threadIdx.x;
    double pc = 0.0;
    if (c < vocab) {
      const float v = val(c);
      if (kept(v)) pc = (double)__fdiv_rn(expf(v - mx), s2);
    }
    // inclusive scan of pc across the CTA
    __shared__ double scan[kThreads];
    scan[threadIdx.x] = pc;
    __syncthreads();
    for (int o = 1; o < kThreads; o <<= 1) {
      const double add = threadIdx.x >= o ? scan[threadIdx.x - o] : 0.0;
      __syncthreads();
      scan[threadIdx.x] += add;
      __syncthreads();
    }
    const double cdf = carry_s + scan[threadIdx.x];
    const double prev = cdf - pc;
    if (c < vocab && pc > 0.0 && prev <= u && u < cdf) atomicCAS(&pick_s, -1, c);
    __syncthreads();
    if (threadIdx.x == 0) carry_s += scan[kThreads - 1];
    __syncthreads();
    if (pick_s >= 0) break;
  }
  if (threadIdx.x == 0) {
    int pk = pick_s;
    if (pk < 0) {  // u at the very top after rounding: the last kept token
      pk = 0;
      for (int c = vocab - 1; c >= 0; --c)
        if (kept(val(c))) { pk = c; break; }
    }
    out[r] = pk;
  }
}

}  // namespace

int sample_greedy(const float* logits, int rows_cap, const int32_t* rows_dev, int vocab, int ld,
                  const uint8_t* eos_mask, int eos_id, const float* penalty, const uint32_t* seen,
                  int32_t* out, cudaStream_t st) {
  if (rows_cap <= 0) return VLLT_OK;
  VLLT_REQUIRE(vocab > 0 && ld >= vocab, "sample_greedy: bad vocab/ld");
  greedy_kernel<<<rows_cap, kThreads, 0, st>>>(logits, vocab, ld, eos_mask, eos_id, penalty, seen,
                                               (vocab + 31) / 32, rows_cap, rows_dev, out);
  return check_launch("sample_greedy");
}

int spec_accept(const int32_t* cu_rows, const int32_t* drafts, const int32_t* draft_off,
                int num_seqs, const int32_t* picks, int32_t* n_accepted, cudaStream_t st) {
  if (num_seqs <= 0) return VLLT_OK;
  accept_kernel<<<ceil_div(num_seqs, 128), 128, 0, st>>>(cu_rows, drafts, draft_off, num_seqs, picks, n_accepted);
  return check_launch("spec_accept");
}

int sample_top_p(const float* logits, int rows, int vocab, int ld, int logit_rows, const int32_t* row_index,
                 const uint8_t* eos_mask, int eos_id, const float* penalty, const uint32_t* seen,
                 const float* temperature, const int32_t* top_k, const float* top_p, const double* u,
                 int32_t* out, cudaStream_t st) {
  if (rows <= 0) return VLLT_OK;
  VLLT_REQUIRE(vocab > 0 && ld >= vocab && logit_rows > 0 && temperature && u, "sample_top_p: bad arguments");
  top_p_kernel<<<rows, kThreads, 0, st>>>(logits, vocab, ld, logit_rows, row_index, eos_mask, eos_id, penalty,
                                          seen, (vocab + 31) / 32, temperature, top_k, top_p, u, out);
  return check_launch("sample_top_p");
}

}  // namespace vllt
