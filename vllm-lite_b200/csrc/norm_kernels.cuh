// Device code of the row-wise kernels (launched by norm.cu): RMSNorm, token
// embedding, RoPE, the bf16 model's fused add + RMSNorm, per-row argmax.
// Plain CUDA C++ with no inline PTX beyond device_common.cuh's helpers, so
// the CPU tests can also run it on the host (tests/simt_host.h).
#pragma once

#include <stdint.h>

#include "device_common.cuh"

namespace vllt {
namespace nk {

// One warp per output row. out = x / sqrt(mean(x^2) + eps) * w, the order of
// vllmlite/model.py:17-19 (a true division and a true square root; no rsqrt).
__global__ void rmsnorm_kernel(const float* __restrict__ x, const int32_t* __restrict__ idx,
                               const float* __restrict__ w, float* __restrict__ out, int rows_cap,
                               const int32_t* __restrict__ rows_dev, int dim, float eps) {
  const int rows = rows_dev ? min(*rows_dev, rows_cap) : rows_cap;
  const int r = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (r >= rows) return;
  const int src = idx ? idx[r] : r;
  const float* xr = x + (int64_t)src * dim;
  float ss = 0.f;
  for (int c = lane * 4; c < dim; c += 128) {
    const float4 v = *reinterpret_cast<const float4*>(xr + c);
    ss = fmaf(v.x, v.x, ss);
    ss = fmaf(v.y, v.y, ss);
    ss = fmaf(v.z, v.z, ss);
    ss = fmaf(v.w, v.w, ss);
  }
  ss = warp_sum(ss);
  const float denom = sqrtf(__fadd_rn(__fdiv_rn(ss, (float)dim), eps));
  float* orow = out + (int64_t)r * dim;
  for (int c = lane * 4; c < dim; c += 128) {
    const float4 v = *reinterpret_cast<const float4*>(xr + c);
    const float4 g = *reinterpret_cast<const float4*>(w + c);
    float4 o;
    o.x = __fmul_rn(__fdiv_rn(v.x, denom), g.x);
    o.y = __fmul_rn(__fdiv_rn(v.y, denom), g.y);
    o.z = __fmul_rn(__fdiv_rn(v.z, denom), g.z);
    o.w = __fmul_rn(__fdiv_rn(v.w, denom), g.w);
    *reinterpret_cast<float4*>(orow + c) = o;
  }
}

// x[t] = emb[token[t]] (vllmlite/model.py:93). Out-of-range ids give zeros.
__global__ void embed_kernel(const float* __restrict__ emb, const int32_t* __restrict__ tok,
                             float* __restrict__ x, int T_cap, const int32_t* __restrict__ T_dev,
                             int dim, int vocab) {
  const int T = T_dev ? min(*T_dev, T_cap) : T_cap;
  const int vec = dim / 4;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < (int64_t)T * vec;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int t = (int)(i / vec), c = (int)(i % vec) * 4;
    const int id = tok[t];
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (id >= 0 && id < vocab) v = *reinterpret_cast<const float4*>(emb + (int64_t)id * dim + c);
    *reinterpret_cast<float4*>(x + (int64_t)t * dim + c) = v;
  }
}

// In-place interleaved-pair rotation (vllmlite/attention.py:28-37).
__global__ void rope_kernel(float* __restrict__ x, const int32_t* __restrict__ positions,
                            const float* __restrict__ cos_t, const float* __restrict__ sin_t,
                            int T, int heads, int D, int max_pos) {
  const int half = D / 2;
  const int64_t total = (int64_t)T * heads * half;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int pi = (int)(i % half);
    const int64_t th = i / half;
    const int t = (int)(th / heads);
    const int p = min(max(positions[t], 0), max_pos - 1);
    const float c = cos_t[(int64_t)p * half + pi], s = sin_t[(int64_t)p * half + pi];
    float* e = x + th * D + 2 * pi;
    const float x1 = e[0], x2 = e[1];
    e[0] = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s));
    e[1] = __fadd_rn(__fmul_rn(x1, s), __fmul_rn(x2, c));
  }
}

// x[t] = float(emb_bf16[token[t]]) (bf16 model; vllmlite/model.py:93).
__global__ void embed_bf16_kernel(const __nv_bfloat16* __restrict__ emb, const int32_t* __restrict__ tok,
                                  float* __restrict__ x, int T_cap, const int32_t* __restrict__ T_dev, int dim,
                                  int vocab) {
  const int T = T_dev ? min(*T_dev, T_cap) : T_cap;
  const int vec = dim / 8;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < (int64_t)T * vec;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int t = (int)(i / vec), c = (int)(i % vec) * 8;
    const int id = tok[t];
    float* dst = x + (int64_t)t * dim + c;
    if (id < 0 || id >= vocab) {
      *reinterpret_cast<float4*>(dst) = make_float4(0.f, 0.f, 0.f, 0.f);
      *reinterpret_cast<float4*>(dst + 4) = make_float4(0.f, 0.f, 0.f, 0.f);
      continue;
    }
    const uint4 w = *reinterpret_cast<const uint4*>(emb + (int64_t)id * dim + c);
    *reinterpret_cast<float4*>(dst) = make_float4(__uint_as_float(w.x << 16), __uint_as_float(w.x & 0xffff0000u),
                                                  __uint_as_float(w.y << 16), __uint_as_float(w.y & 0xffff0000u));
    *reinterpret_cast<float4*>(dst + 4) = make_float4(__uint_as_float(w.z << 16), __uint_as_float(w.z & 0xffff0000u),
                                                      __uint_as_float(w.w << 16), __uint_as_float(w.w & 0xffff0000u));
  }
}

// One CTA (256 threads) per row of the bf16 model: optionally x += add (the
// all-reduced partial of a tensor-parallel projection, written back), then
// out = bf16(x / sqrt(mean(x^2) + eps) * w). idx gathers rows (logit rows).
__global__ void rmsnorm_bf16_kernel(float* __restrict__ x, const __nv_bfloat16* __restrict__ add,
                                    const int32_t* __restrict__ idx, const float* __restrict__ w,
                                    __nv_bfloat16* __restrict__ out, int rows_cap,
                                    const int32_t* __restrict__ rows_dev, int dim, float eps) {
  pdl_trigger();  // the projection that reads `out` may start its set-up (it waits for this grid)
  const int rows = rows_dev ? min(*rows_dev, rows_cap) : rows_cap;
  const int r = blockIdx.x;
  if (r >= rows) return;
  const int src = idx ? idx[r] : r;
  float* xr = x + (int64_t)src * dim;
  float ss = 0.f;
  for (int c = threadIdx.x * 4; c < dim; c += blockDim.x * 4) {
    float4 v = *reinterpret_cast<const float4*>(xr + c);
    if (add) {
      const uint2 a = *reinterpret_cast<const uint2*>(add + (int64_t)src * dim + c);
      v.x += __uint_as_float(a.x << 16); v.y += __uint_as_float(a.x & 0xffff0000u);
      v.z += __uint_as_float(a.y << 16); v.w += __uint_as_float(a.y & 0xffff0000u);
      *reinterpret_cast<float4*>(xr + c) = v;
    }
    ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
  }
  __shared__ float red[8];
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (int)(blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    t = warp_sum(t);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  const float inv = rsqrtf(red[0] / (float)dim + eps);
  __nv_bfloat16* orow = out + (int64_t)r * dim;
  for (int c = threadIdx.x * 4; c < dim; c += blockDim.x * 4) {
    const float4 v = *reinterpret_cast<const float4*>(xr + c);
    const float4 g = *reinterpret_cast<const float4*>(w + c);
    const __nv_bfloat162 a = __floats2bfloat162_rn(v.x * inv * g.x, v.y * inv * g.y);
    const __nv_bfloat162 b = __floats2bfloat162_rn(v.z * inv * g.z, v.w * inv * g.w);
    uint2 o;
    o.x = *reinterpret_cast<const uint32_t*>(&a);
    o.y = *reinterpret_cast<const uint32_t*>(&b);
    *reinterpret_cast<uint2*>(orow + c) = o;
  }
}

// Per row: (max value, first index of the max) over [0, vocab); index + offset.
__global__ void argmax_rows_kernel(const float* __restrict__ logits, int vocab, int ld, int offset,
                                   int rows_cap, const int32_t* __restrict__ rows_dev, float* __restrict__ val,
                                   int32_t* __restrict__ idx) {
  const int rows = rows_dev ? min(*rows_dev, rows_cap) : rows_cap;
  const int r = blockIdx.x;
  if (r >= rows) return;
  const float* x = logits + (int64_t)r * ld;
  float bv = -INFINITY;
  int bi = INT32_MAX;
  if (((uintptr_t)x & 15) == 0) {
    row_argmax_part(x, vocab, threadIdx.x, blockDim.x, bv, bi);
  } else {
    for (int c = threadIdx.x; c < vocab; c += blockDim.x) {
      const float v = x[c];
      if (v > bv || (v == bv && c < bi)) { bv = v; bi = c; }
    }
  }
  __shared__ float sv[32];
  __shared__ int si[32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
  }
  if ((threadIdx.x & 31) == 0) { sv[threadIdx.x >> 5] = bv; si[threadIdx.x >> 5] = bi; }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
      if (sv[w] > bv || (sv[w] == bv && si[w] < bi)) { bv = sv[w]; bi = si[w]; }
    val[r] = bv;
    idx[r] = bi == INT32_MAX ? offset : bi + offset;
  }
}

}  // namespace nk
}  // namespace vllt
