// fp32 SIMT GEMM with fused epilogues (parity mode: true fp32, no TF32).
//
// C[M][N] = A[M][K] @ B[K][N], both row-major (the reference's [in][out]
// weights, vllmlite/model.py:34-43). Register-blocked FFMA tiles, double-
// buffered through shared memory. The epilogue functor receives TN
// consecutive output columns of one row.
#pragma once

#include "common.cuh"

namespace vllt {

template <int BM, int BN, int TM, int TN, class Epi>
__global__ void __launch_bounds__(256) sgemm_kernel(const float* __restrict__ A, int lda,
                                                    const float* __restrict__ B, int ldb,
                                                    int M_cap, const int* __restrict__ M_dev,
                                                    int N, int K, Epi epi) {
  constexpr int BK = 16;
  constexpr int TX = BN / TN, TY = BM / TM;
  static_assert(TX * TY == 256, "256 threads");
  constexpr int A_VEC = BM * BK / 4;
  constexpr int A_PER = (A_VEC + 255) / 256;
  constexpr int B_VEC = BK * BN / 4;
  constexpr int B_PER = (B_VEC + 255) / 256;
  __shared__ __align__(16) float As[2][BK][BM];
  __shared__ __align__(16) float Bs[2][BK][BN];

  const int M = M_dev ? min(*M_dev, M_cap) : M_cap;
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
  if (m0 >= M) return;
  const int tid = threadIdx.x, tx = tid % TX, ty = tid / TX;

  float4 a_reg[A_PER], b_reg[B_PER];
  auto load = [&](int k0) {
#pragma unroll
    for (int i = 0; i < A_PER; ++i) {
      const int v = tid + i * 256;
      float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
      if (v < A_VEC) {
        const int r = v / (BK / 4), c = (v % (BK / 4)) * 4;
        const int gm = m0 + r, gk = k0 + c;
        if (gm < M && gk < K) x = *reinterpret_cast<const float4*>(A + (int64_t)gm * lda + gk);
      }
      a_reg[i] = x;
    }
#pragma unroll
    for (int i = 0; i < B_PER; ++i) {
      const int v = tid + i * 256;
      float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
      if (v < B_VEC) {
        const int r = v / (BN / 4), c = (v % (BN / 4)) * 4;
        const int gk = k0 + r, gn = n0 + c;
        if (gk < K && gn < N) x = *reinterpret_cast<const float4*>(B + (int64_t)gk * ldb + gn);
      }
      b_reg[i] = x;
    }
  };
  auto store = [&](int buf) {
#pragma unroll
    for (int i = 0; i < A_PER; ++i) {
      const int v = tid + i * 256;
      if (v < A_VEC) {
        const int r = v / (BK / 4), c = (v % (BK / 4)) * 4;
        As[buf][c + 0][r] = a_reg[i].x;
        As[buf][c + 1][r] = a_reg[i].y;
        As[buf][c + 2][r] = a_reg[i].z;
        As[buf][c + 3][r] = a_reg[i].w;
      }
    }
#pragma unroll
    for (int i = 0; i < B_PER; ++i) {
      const int v = tid + i * 256;
      if (v < B_VEC) {
        const int r = v / (BN / 4), c = (v % (BN / 4)) * 4;
        *reinterpret_cast<float4*>(&Bs[buf][r][c]) = b_reg[i];
      }
    }
  };

  float acc[TM][TN];
#pragma unroll
  for (int i = 0; i < TM; ++i)
#pragma unroll
    for (int j = 0; j < TN; ++j) acc[i][j] = 0.f;

  load(0);
  store(0);
  __syncthreads();
  for (int k0 = 0, it = 0; k0 < K; k0 += BK, ++it) {
    const int cur = it & 1;
    const bool more = k0 + BK < K;
    if (more) load(k0 + BK);
#pragma unroll
    for (int kk = 0; kk < BK; ++kk) {
      float a[TM], b[TN];
#pragma unroll
      for (int i = 0; i < TM; ++i) a[i] = As[cur][kk][ty * TM + i];
#pragma unroll
      for (int j = 0; j < TN; ++j) b[j] = Bs[cur][kk][tx * TN + j];
#pragma unroll
      for (int i = 0; i < TM; ++i)
#pragma unroll
        for (int j = 0; j < TN; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    if (more) store(cur ^ 1);
    __syncthreads();
  }

  const int col = n0 + tx * TN;
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

// Tile choice by the row capacity of the launch.
template <class Epi>
int sgemm_launch(const float* A, int lda, const float* B, int ldb, int M_cap, const int* M_dev,
                 int N, int K, const Epi& epi, cudaStream_t st) {
  if (M_cap <= 0) return VLLT_OK;
  VLLT_REQUIRE(K % 4 == 0 && N % 4 == 0 && lda % 4 == 0 && ldb % 4 == 0,
               "sgemm: K, N and leading dims must be multiples of 4 (K=%d N=%d)", K, N);
  VLLT_REQUIRE(((uintptr_t)A % 16) == 0 && ((uintptr_t)B % 16) == 0, "sgemm: operands must be 16-byte aligned");
  constexpr int BN = 64;
  const int gx = ceil_div(N, BN);
  if (M_cap <= 16) {
    sgemm_kernel<16, BN, 1, 4, Epi><<<dim3(gx, ceil_div(M_cap, 16)), 256, 0, st>>>(A, lda, B, ldb, M_cap, M_dev, N, K, epi);
  } else if (M_cap <= 32) {
    sgemm_kernel<32, BN, 2, 4, Epi><<<dim3(gx, ceil_div(M_cap, 32)), 256, 0, st>>>(A, lda, B, ldb, M_cap, M_dev, N, K, epi);
  } else if (M_cap <= 256) {
    sgemm_kernel<64, BN, 4, 4, Epi><<<dim3(gx, ceil_div(M_cap, 64)), 256, 0, st>>>(A, lda, B, ldb, M_cap, M_dev, N, K, epi);
  } else {
    sgemm_kernel<128, BN, 8, 4, Epi><<<dim3(gx, ceil_div(M_cap, 128)), 256, 0, st>>>(A, lda, B, ldb, M_cap, M_dev, N, K, epi);
  }
  return check_launch("sgemm");
}

}  // namespace vllt
