// fp32 SIMT GEMM with fused epilogues (parity mode: true fp32, no TF32).
//
// C[M][N] = A[M][K] @ B[K][N], both row-major (the reference's [in][out]
// weights, vllmlite/model.py:34-43). Register-blocked FFMA tiles fed by a
// 3-stage cp.async pipeline (BK = 32).
//
// Decode steps have few rows (M ~ batch), so one CTA per output tile would
// walk all of K serially with a handful of CTAs on 148 SMs: latency bound.
// For small M the K range is split across CTAs (grid.z). Every slice writes
// its partial tile to a workspace; the last slice to finish (an atomic
// counter per tile) sums the partials in slice order -- deterministic -- runs
// the epilogue and resets the counter, so the kernel can be replayed from a
// CUDA graph.
#pragma once

#include <algorithm>

#include "common.cuh"
#include "gemm_f32_kernels.cuh"

namespace vllt {

template <int BM, int BN, int BK, int TM, int TN, int THREADS, class Epi>
int sgemm_go(const float* A, int lda, const float* B, int ldb, int M_cap, const int* M_dev, int N, int K,
             const Epi& epi, const GemmScratch* sc, cudaStream_t st) {
  const int k_slice = gemm_k_slice(M_cap, N, K, BM, BN, BK, sc);
  const int ks = ceil_div(K, k_slice);
  dim3 grid(ceil_div(N, BN), ceil_div(M_cap, BM), ks);
  VLLT_LAUNCH(grid, THREADS, 0, st, sgemm_kernel<BM, BN, BK, TM, TN, THREADS, Epi>)(
      A, lda, B, ldb, M_cap, M_dev, N, K, k_slice, ks > 1 ? sc->partials : nullptr,
      ks > 1 ? sc->counters : nullptr, epi);
  return check_launch("sgemm");
}

// Tile choice by the row capacity of the launch.
template <class Epi>
int sgemm_launch(const float* A, int lda, const float* B, int ldb, int M_cap, const int* M_dev,
                 int N, int K, const Epi& epi, cudaStream_t st, const GemmScratch* sc = nullptr) {
  if (M_cap <= 0) return VLLT_OK;
  VLLT_REQUIRE(K % 4 == 0 && N % 4 == 0 && lda % 4 == 0 && ldb % 4 == 0,
               "sgemm: K, N and leading dims must be multiples of 4 (K=%d N=%d)", K, N);
  VLLT_REQUIRE(((uintptr_t)A % 16) == 0 && ((uintptr_t)B % 16) == 0, "sgemm: operands must be 16-byte aligned");
  if (M_cap <= 16) return sgemm_go<16, 64, 32, 2, 4, 128>(A, lda, B, ldb, M_cap, M_dev, N, K, epi, sc, st);
  if (M_cap <= 32) return sgemm_go<32, 64, 32, 4, 4, 128>(A, lda, B, ldb, M_cap, M_dev, N, K, epi, sc, st);
  if (M_cap <= 64) return sgemm_go<64, 64, 16, 4, 4, 256>(A, lda, B, ldb, M_cap, M_dev, N, K, epi, sc, st);
  return sgemm_go<128, 64, 16, 8, 4, 256>(A, lda, B, ldb, M_cap, M_dev, N, K, epi, sc, st);
}

}  // namespace vllt
