// Epilogues of the bf16 tensor-core GEMMs (gemm_bf16_tc.cuh): what one
// call does with 32 consecutive fp32 accumulator columns of one row. Plain
// CUDA C++, so the CPU tests can also run them on the host.
#pragma once

#include <stdint.h>

#include "device_common.cuh"

namespace vllt {

// ---- bf16-path epilogues (32 consecutive columns per call) --------------------------

struct EpiStoreF32 {  // C fp32 [M][ldc], columns < n_valid
  float* C;
  int ldc, n_valid;
  template <int TN> __device__ void apply(int row, int col, const float (&v)[TN]) const {
    float* dst = C + (int64_t)row * ldc + col;
    if (col + TN <= n_valid && ((ldc | col) & 3) == 0) {
#pragma unroll
      for (int j = 0; j < TN; j += 4) *reinterpret_cast<float4*>(dst + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
    } else {
#pragma unroll
      for (int j = 0; j < TN; ++j)
        if (col + j < n_valid) dst[j] = v[j];
    }
  }
};

struct EpiStoreBF16 {  // C bf16 [M][ldc], columns < n_valid
  __nv_bfloat16* C;
  int ldc, n_valid;
  template <int TN> __device__ void apply(int row, int col, const float (&v)[TN]) const {
    __nv_bfloat16* dst = C + (int64_t)row * ldc + col;
#pragma unroll
    for (int j = 0; j < TN; ++j)
      if (col + j < n_valid) dst[j] = __float2bfloat16_rn(v[j]);
  }
};

}  // namespace vllt

namespace vllt {

// x[row][col..] += acc (fp32 residual stream; tensor-parallel size 1)
struct EpiResidualF32 {
  float* x;
  int ld;
  template <int TN> __device__ void apply(int row, int col, const float (&v)[TN]) const {
    float* dst = x + (int64_t)row * ld + col;
#pragma unroll
    for (int j = 0; j < TN; j += 4) {
      float4 o = *reinterpret_cast<float4*>(dst + j);
      o.x += v[j]; o.y += v[j + 1]; o.z += v[j + 2]; o.w += v[j + 3];
      *reinterpret_cast<float4*>(dst + j) = o;
    }
  }
};

// columns interleaved (gate_j, up_j) -> act[row][col/2 + j] = silu(gate_j) * up_j, bf16
struct EpiSwiGLUBF16 {
  __nv_bfloat16* act;
  int ld;
  template <int TN> __device__ void apply(int row, int col, const float (&v)[TN]) const {
    __nv_bfloat16* dst = act + (int64_t)row * ld + col / 2;
#pragma unroll
    for (int j = 0; j < TN / 2; j += 2) {
      const float g0 = v[2 * j], u0 = v[2 * j + 1], g1 = v[2 * j + 2], u1 = v[2 * j + 3];
      const float a0 = g0 / (1.0f + __expf(-g0)) * u0, a1 = g1 / (1.0f + __expf(-g1)) * u1;
      *reinterpret_cast<__nv_bfloat162*>(dst + j) = __floats2bfloat162_rn(a0, a1);
    }
  }
};

// QKV projection (bf16 model): RoPE on q and k columns (interleaved pairs,
// vllmlite/attention.py:28-37), q -> bf16 buffer, k and v -> bf16 paged cache
// at the token's slot. 32 columns never straddle a head (head_dim % 32 == 0).
struct EpiQKVBF16 {
  __nv_bfloat16* q_out;  // [T][H*D]
  __nv_bfloat16* kc;     // layer base [NB][n_kv][bs][D]
  __nv_bfloat16* vc;
  const int32_t* pos;
  const int32_t* slot;
  const float* cos_t;    // [max_pos][D/2]
  const float* sin_t;
  int H, n_kv, D, bs, max_pos;
  int64_t num_slots;
  template <int TN> __device__ void apply(int row, int col, const float (&v)[TN]) const {
    const int qw = H * D, kw = n_kv * D;
    float o[TN];
    if (col < qw + kw) {
      const int d0 = col % D;
      const int p = min(max(pos[row], 0), max_pos - 1);
      const float* cr = cos_t + (int64_t)p * (D / 2) + d0 / 2;
      const float* sr = sin_t + (int64_t)p * (D / 2) + d0 / 2;
#pragma unroll
      for (int j = 0; j < TN; j += 2) {
        const float c = cr[j / 2], s = sr[j / 2];
        o[j] = v[j] * c - v[j + 1] * s;
        o[j + 1] = v[j] * s + v[j + 1] * c;
      }
    } else {
#pragma unroll
      for (int j = 0; j < TN; ++j) o[j] = v[j];
    }
    __nv_bfloat16* dst;
    if (col < qw) {
      dst = q_out + (int64_t)row * qw + col;
    } else {
      const int64_t sl = slot[row];
      if (sl < 0 || sl >= num_slots) return;
      const int64_t blk = sl / bs, off = sl % bs;
      const bool is_k = col < qw + kw;
      const int c = col - qw - (is_k ? 0 : kw);
      dst = (is_k ? kc : vc) + ((blk * n_kv + c / D) * bs + off) * D + c % D;
    }
#pragma unroll
    for (int j = 0; j < TN; j += 8) {
      uint4 w;
      __nv_bfloat162 t0 = __floats2bfloat162_rn(o[j], o[j + 1]), t1 = __floats2bfloat162_rn(o[j + 2], o[j + 3]);
      __nv_bfloat162 t2 = __floats2bfloat162_rn(o[j + 4], o[j + 5]), t3 = __floats2bfloat162_rn(o[j + 6], o[j + 7]);
      w.x = *reinterpret_cast<uint32_t*>(&t0); w.y = *reinterpret_cast<uint32_t*>(&t1);
      w.z = *reinterpret_cast<uint32_t*>(&t2); w.w = *reinterpret_cast<uint32_t*>(&t3);
      *reinterpret_cast<uint4*>(dst + j) = w;
    }
  }
};

}  // namespace vllt
