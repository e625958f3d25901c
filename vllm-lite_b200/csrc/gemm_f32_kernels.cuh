// Device code of the fp32 SIMT GEMM and its fused epilogues (launched
// through gemm_f32.cuh). Plain CUDA C++ with no inline PTX beyond
// device_common.cuh's helpers, so the CPU tests can also run it on the host
// (tests/simt_host.h).
#pragma once

#include <stdint.h>

#include "device_common.cuh"

namespace vllt {

constexpr int kGemmStages = 3;

template <int BM, int BN, int BK, int TM, int TN, int THREADS, class Epi>
__global__ void __launch_bounds__(THREADS) sgemm_kernel(const float* __restrict__ A, int lda,
                                                        const float* __restrict__ B, int ldb,
                                                        int M_cap, const int* __restrict__ M_dev,
                                                        int N, int K, int k_slice,
                                                        float* __restrict__ ws, int* __restrict__ counters,
                                                        Epi epi) {
  constexpr int NS = kGemmStages;
  constexpr int TX = BN / TN, TY = BM / TM;
  static_assert(TX * TY == THREADS, "thread tile");
  constexpr int AST = BK + 4;  // A tile row stride (floats), keeps 16-byte alignment
  constexpr int A_CH = BM * BK / 4, B_CH = BK * BN / 4;  // 16-byte chunks per stage
  __shared__ __align__(16) float As[NS][BM * AST];
  __shared__ __align__(16) float Bs[NS][BK * BN];
  __shared__ int s_last;

  const int M = M_dev ? min(*M_dev, M_cap) : M_cap;
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
  if (m0 >= M) return;
  const int tid = threadIdx.x, tx = tid % TX, ty = tid / TX;
  const int ks = gridDim.z, z = blockIdx.z;
  const int kb = z * k_slice, ke = min(K, kb + k_slice);
  const int nk = (ke - kb + BK - 1) / BK;

  auto load_stage = [&](int stage, int k0) {
#pragma unroll
    for (int i = tid; i < A_CH; i += THREADS) {
      const int r = i / (BK / 4), c = (i % (BK / 4)) * 4;
      const int gm = m0 + r, gk = k0 + c;
      const bool ok = gm < M && gk < ke;
      cp_async16(&As[stage][r * AST + c], ok ? (const void*)(A + (int64_t)gm * lda + gk) : (const void*)A, ok);
    }
#pragma unroll
    for (int i = tid; i < B_CH; i += THREADS) {
      const int r = i / (BN / 4), c = (i % (BN / 4)) * 4;
      const int gk = k0 + r, gn = n0 + c;
      const bool ok = gk < ke && gn < N;
      cp_async16(&Bs[stage][r * BN + c], ok ? (const void*)(B + (int64_t)gk * ldb + gn) : (const void*)B, ok);
    }
  };

  float acc[TM][TN];
#pragma unroll
  for (int i = 0; i < TM; ++i)
#pragma unroll
    for (int j = 0; j < TN; ++j) acc[i][j] = 0.f;

#pragma unroll
  for (int s = 0; s < NS - 1; ++s) {
    if (s < nk) load_stage(s, kb + s * BK);
    cp_async_commit();
  }
  for (int it = 0; it < nk; ++it) {
    cp_async_wait<NS - 2>();
    __syncthreads();
    const int nxt = it + NS - 1;
    if (nxt < nk) load_stage(nxt % NS, kb + nxt * BK);
    cp_async_commit();
    const float* as = As[it % NS];
    const float* bs = Bs[it % NS];
#pragma unroll
    for (int kk = 0; kk < BK; ++kk) {
      float a[TM], b[TN];
#pragma unroll
      for (int i = 0; i < TM; ++i) a[i] = as[(ty * TM + i) * AST + kk];
#pragma unroll
      for (int j = 0; j < TN; j += 4) {
        const float4 v = *reinterpret_cast<const float4*>(&bs[kk * BN + tx * TN + j]);
        b[j] = v.x; b[j + 1] = v.y; b[j + 2] = v.z; b[j + 3] = v.w;
      }
#pragma unroll
      for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
  }
  cp_async_wait<0>();

  const int col = n0 + tx * TN;
  if (ks > 1) {
    // partial tile -> workspace; the last slice reduces in slice order
    const int tile = blockIdx.y * gridDim.x + blockIdx.x;
    float* mine = ws + ((int64_t)tile * ks + z) * (BM * BN);
#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
      for (int j = 0; j < TN; j += 4)
        *reinterpret_cast<float4*>(&mine[(ty * TM + i) * BN + tx * TN + j]) =
            make_float4(acc[i][j], acc[i][j + 1], acc[i][j + 2], acc[i][j + 3]);
    __threadfence();
    __syncthreads();
    if (tid == 0) s_last = atomicAdd(&counters[tile], 1) == ks - 1;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    const float* base = ws + (int64_t)tile * ks * (BM * BN);
#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
      for (int j = 0; j < TN; ++j) acc[i][j] = 0.f;
    for (int zz = 0; zz < ks; ++zz) {
      const float* part = base + (int64_t)zz * (BM * BN);
#pragma unroll
      for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN; j += 4) {
          const float4 v = __ldcg(reinterpret_cast<const float4*>(&part[(ty * TM + i) * BN + tx * TN + j]));
          acc[i][j] += v.x; acc[i][j + 1] += v.y; acc[i][j + 2] += v.z; acc[i][j + 3] += v.w;
        }
    }
    if (tid == 0) counters[tile] = 0;  // ready for the next launch / graph replay
  }
  if (col >= N) return;
#pragma unroll
  for (int i = 0; i < TM; ++i) {
    const int row = m0 + ty * TM + i;
    if (row < M) epi.template apply<TN>(row, col, acc[i]);
  }
}

// ---- epilogues ---------------------------------------------------------------

struct EpiStore {  // C = acc, columns < n_valid stored
  float* C;
  int ldc, n_valid;
  template <int TN> __device__ void apply(int row, int col, const float (&v)[TN]) const {
#pragma unroll
    for (int j = 0; j < TN; ++j)
      if (col + j < n_valid) C[(int64_t)row * ldc + col + j] = v[j];
  }
};

struct EpiResidual {  // C += acc (x = x + y @ W, vllmlite/model.py:114, :117)
  float* C;
  int ldc;
  template <int TN> __device__ void apply(int row, int col, const float (&v)[TN]) const {
#pragma unroll
    for (int j = 0; j < TN; ++j) C[(int64_t)row * ldc + col + j] += v[j];
  }
};

struct EpiSwiGLU {  // columns interleaved (gate_j, up_j): out_j = silu(gate_j) * up_j
  float* out;
  int ldo;
  template <int TN> __device__ void apply(int row, int col, const float (&v)[TN]) const {
#pragma unroll
    for (int j = 0; j < TN / 2; ++j) {
      const float g = v[2 * j], u = v[2 * j + 1];
      const float sg = __fdiv_rn(g, __fadd_rn(1.0f, expf(-g)));  // model.py:22-23
      out[(int64_t)row * ldo + col / 2 + j] = __fmul_rn(sg, u);
    }
  }
};

// QKV projection epilogue: RoPE on the q and k columns (interleaved pairs,
// vllmlite/attention.py:28-37), q to its buffer, k and v straight into the paged
// cache at the token's slot (write_kv, attention.py:47-49).
struct EpiQKV {
  float* q_out;            // [T][H*D]
  float* kc;               // layer base [NB][n_kv][bs][D]
  float* vc;
  const int32_t* pos;      // [T]
  const int32_t* slot;     // [T]
  const float* cos_t;      // [max_pos][D/2]
  const float* sin_t;
  int H, n_kv, D, bs, max_pos;
  int64_t num_slots;
  template <int TN> __device__ void apply(int row, int col, const float (&v)[TN]) const {
    const int qw = H * D, kw = n_kv * D;
    float o[TN];
    const bool rot = col < qw + kw;
    if (rot) {
      const int d0 = col % D;
      const int p = min(max(pos[row], 0), max_pos - 1);
#pragma unroll
      for (int j = 0; j < TN; j += 2) {
        const int i = (d0 + j) >> 1;
        const float c = cos_t[(int64_t)p * (D / 2) + i], s = sin_t[(int64_t)p * (D / 2) + i];
        const float x1 = v[j], x2 = v[j + 1];
        o[j] = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s));
        o[j + 1] = __fadd_rn(__fmul_rn(x1, s), __fmul_rn(x2, c));
      }
    } else {
#pragma unroll
      for (int j = 0; j < TN; ++j) o[j] = v[j];
    }
    if (col < qw) {
#pragma unroll
      for (int j = 0; j < TN; ++j) q_out[(int64_t)row * qw + col + j] = o[j];
      return;
    }
    const int64_t sl = slot[row];
    if (sl < 0 || sl >= num_slots) return;
    const int64_t blk = sl / bs, off = sl % bs;
    const bool is_k = col < qw + kw;
    const int c = col - qw - (is_k ? 0 : kw);
    const int h = c / D, d = c % D;
    float* dst = (is_k ? kc : vc) + ((blk * n_kv + h) * bs + off) * D + d;
#pragma unroll
    for (int j = 0; j < TN; ++j) dst[j] = o[j];
  }
};

// Split-K scratch for the small-M path: partial tiles and per-tile counters.
struct GemmScratch {
  float* partials;
  int* counters;        // zeroed once; every reducer resets its own
  int64_t partial_floats;
  int n_counters;
};

// K slice length: whole K unless M is small; then ~4 k-steps per slice, at
// most 8 slices, and never more partial floats / counters than the scratch has.
inline int gemm_k_slice(int M_cap, int N, int K, int BM, int BN, int BK, const GemmScratch* sc) {
  if (!sc || M_cap > 64) return K;
  const int tiles = ceil_div(N, BN) * ceil_div(M_cap, BM);
  int ks = min(8, ceil_div(K, 4 * BK));
  while (ks > 1 && ((int64_t)tiles * ks * BM * BN > sc->partial_floats || tiles > sc->n_counters)) --ks;
  if (ks <= 1) return K;
  return ceil_div(ceil_div(K, ks), BK) * BK;
}

// Scratch the split-K path may use for up to 64 rows and N columns.
inline int64_t gemm_scratch_floats(int N) { return (int64_t)ceil_div(N, 64) * 64 * 64 * 8; }
inline int gemm_scratch_counters(int N) { return ceil_div(N, 64) * 4; }

}  // namespace vllt
