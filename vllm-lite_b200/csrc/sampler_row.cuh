// The temperature branch of vllm-lite's sample() (vllmlite/sampling.py:41-64)
// for one row of logits, written once for the device kernel (top_p_kernel in
// sampling.cu, one CTA per row) and for the host-compiled CPU tests, which run
// this same code on the reference's fixtures. The parallel parts (reductions
// over the vocabulary, the cumulative-distribution search) are left to an
// execution policy: a CTA's block reductions and scan on the device, plain
// loops on the host.
//
// Order of the steps, as the reference: EOS masked to -inf while min_tokens
// is not reached (:51-52), the repetition penalty on every seen token (:54,
// :8-13), division by the temperature (:59), top-k (:16-20), top-p (:23-33),
// softmax (:63) and numpy's Generator.choice (:64). The k-th largest value and
// the nucleus threshold are found by bisection over float order keys, so any
// vocabulary size works with O(32 * vocab) work and no sort. The draw takes
// the uniform the request's generator would hand choice(): the first index
// whose float64 CDF (cumulative sum of the kept probabilities, divided by the
// total) exceeds it.
#pragma once

#include <math.h>
#include <stdint.h>
#include <string.h>

#ifndef __CUDACC__
#ifndef __host__
#define __host__
#endif
#ifndef __device__
#define __device__
#endif
#endif

namespace vllt {
namespace sampler {

__host__ __device__ inline uint32_t float_bits(float f) {
#ifdef __CUDA_ARCH__
  return __float_as_uint(f);
#else
  uint32_t u;
  memcpy(&u, &f, 4);
  return u;
#endif
}

__host__ __device__ inline float bits_float(uint32_t u) {
#ifdef __CUDA_ARCH__
  return __uint_as_float(u);
#else
  float f;
  memcpy(&f, &u, 4);
  return f;
#endif
}

// A float's bits as an unsigned key with the same order (for bisection).
__host__ __device__ inline uint32_t order_key(float f) {
  const uint32_t u = float_bits(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// IEEE round-to-nearest division and product (no contraction into an FMA).
__host__ __device__ inline float div_rn(float a, float b) {
#ifdef __CUDA_ARCH__
  return __fdiv_rn(a, b);
#else
  return a / b;
#endif
}
__host__ __device__ inline float mul_rn(float a, float b) {
#ifdef __CUDA_ARCH__
  return __fmul_rn(a, b);
#else
  return a * b;
#endif
}

// One row of logits seen through the reference's pre-steps (sampling.py:51-59).
struct RowInput {
  const float* x;
  int vocab;
  bool mask_eos;         // min_tokens not reached: EOS -> -inf
  int eos_id;
  float pen;             // repetition penalty
  const uint32_t* seen;  // bitmap of the seen tokens (NULL: no penalty)
  float temp;

  __host__ __device__ float val(int c) const {
    float v = x[c];
    if (mask_eos && c == eos_id) v = -INFINITY;
    if (seen && ((seen[c >> 5] >> (c & 31)) & 1u)) v = v > 0.f ? div_rn(v, pen) : mul_rn(v, pen);
    return div_rn(v, temp);
  }
};

// What a row's draw needs after its reductions: the top-k order-key cut,
// the maximum kept value, the softmax sum over the top-k set, the nucleus
// threshold, and the sums over the final kept set.
struct Thresholds {
  uint32_t cut_key;
  float mx, sum, pmin, p;
  float s2;      // sum of exp(v - mx) over the kept set (float, as the kernel reduces it)
  double total;  // sum of the kept probabilities (float64)
};

// Whether token c survives top-k and top-p (the reference's keep set).
__host__ __device__ inline bool kept(const RowInput& row, const Thresholds& t, float v) {
  return order_key(v) >= t.cut_key && (t.p >= 1.f || div_rn(expf(v - t.mx), t.sum) >= t.pmin);
}

// Probability of token c in the renormalised kept distribution.
__host__ __device__ inline double kept_prob(const RowInput& row, const Thresholds& t, int c) {
  const float v = row.val(c);
  return kept(row, t, v) ? (double)div_rn(expf(v - t.mx), t.s2) : 0.0;
}

// The reductions of one row. P provides: tid() and stride() (this thread's
// slice of the vocabulary) and reduce_sum(int / float / double) and
// reduce_max(float) over all threads.
#ifdef __CUDACC__
#pragma nv_exec_check_disable
#endif
template <class P>
__host__ __device__ Thresholds thresholds(P& pol, const RowInput& row, int k, float p) {
  const int vocab = row.vocab;
  Thresholds t;
  t.p = p;
  // top-k: the largest key v with count(x >= v) >= k
  t.cut_key = 0;
  if (k > 0 && k < vocab) {
    // upper midpoint in 64 bits (lo + (hi - lo + 1) / 2 wraps to lo on the
    // full range and never moves); each step halves [lo, hi], so 32 suffice
    uint32_t lo = 0, hi = 0xffffffffu;
    for (int step = 0; step < 33 && lo < hi; ++step) {
      const uint32_t mid = (uint32_t)(((uint64_t)lo + hi + 1) >> 1);
      int cnt = 0;
      for (int c = pol.tid(); c < vocab; c += pol.stride()) cnt += order_key(row.val(c)) >= mid;
      cnt = pol.reduce_sum(cnt);
      if (cnt >= k) lo = mid; else hi = mid - 1;
    }
    t.cut_key = lo;
  }
  float mx = -INFINITY;
  for (int c = pol.tid(); c < vocab; c += pol.stride()) {
    const float v = row.val(c);
    if (order_key(v) >= t.cut_key) mx = fmaxf(mx, v);
  }
  t.mx = pol.reduce_max(mx);
  float sum = 0.f;
  for (int c = pol.tid(); c < vocab; c += pol.stride()) {
    const float v = row.val(c);
    if (order_key(v) >= t.cut_key) sum += expf(v - t.mx);
  }
  t.sum = pol.reduce_sum(sum);
  // top-p: the smallest probability b with G(b) = sum_{p_j > b} p_j < p; keep p_i >= b
  t.pmin = 0.f;
  if (p < 1.f) {
    uint32_t lo = float_bits(0.f), hi = float_bits(1.f);
    for (int step = 0; step < 33 && lo < hi; ++step) {
      const uint32_t mid = lo + (hi - lo) / 2;
      const float b = bits_float(mid);
      float g = 0.f;
      for (int c = pol.tid(); c < vocab; c += pol.stride()) {
        const float v = row.val(c);
        if (order_key(v) >= t.cut_key) {
          const float pc = div_rn(expf(v - t.mx), t.sum);
          if (pc > b) g += pc;
        }
      }
      g = pol.reduce_sum(g);
      if (g < p) hi = mid; else lo = mid + 1;
    }
    t.pmin = bits_float(lo);
  }
  // renormalised probabilities over the kept set
  float s2 = 0.f;
  for (int c = pol.tid(); c < vocab; c += pol.stride()) {
    const float v = row.val(c);
    if (kept(row, t, v)) s2 += expf(v - t.mx);
  }
  t.s2 = pol.reduce_sum(s2);
  double total = 0.0;
  for (int c = pol.tid(); c < vocab; c += pol.stride()) total += kept_prob(row, t, c);
  t.total = pol.reduce_sum(total);
  return t;
}

// The draw: numpy's choice over the kept distribution (CDF in vocabulary
// order, cumsum in float64 divided by the total, first index with cdf > u).
// P also provides first_crossing(n, pc, u) (the first c with
// cdf(c - 1) <= u < cdf(c), cdf the running sum of pc(c), or -1) and
// last(n, pred) (the largest c with pred(c), or -1).
#ifdef __CUDACC__
#pragma nv_exec_check_disable
#endif
template <class P>
__host__ __device__ int draw(P& pol, const RowInput& row, const Thresholds& t, double uni) {
  int pick = pol.first_crossing(row.vocab, [&](int c) { return kept_prob(row, t, c); }, uni * t.total);
  if (pick < 0)  // u at the very top after rounding: the last kept token
    pick = pol.last(row.vocab, [&](int c) { return kept(row, t, row.val(c)); });
  return pick < 0 ? 0 : pick;
}

// The token sampled for one row.
#ifdef __CUDACC__
#pragma nv_exec_check_disable
#endif
template <class P>
__host__ __device__ int sample_row(P& pol, const RowInput& row, int k, float p, double uni) {
  const Thresholds t = thresholds(pol, row, k, p);
  return draw(pol, row, t, uni);
}

}  // namespace sampler
}  // namespace vllt
