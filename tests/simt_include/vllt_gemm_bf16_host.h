// Test infrastructure: the host build's stand-in for libvllt's tensor-core
// GEMMs (gemm_bf16_tc.cuh), used when forward_bf16.cu is built for the host.
// gemm_bf16_launch computes each row's 32-column chunks of A[M][K] . W[N][K]^T
// from the bf16 operands with fp32 accumulation (columns past N read as zero,
// as the tensor maps' out-of-bounds fill gives the device kernels) and hands
// them to the library's own epilogue (gemm_bf16_epi.cuh). The tcgen05 kernels
// themselves are not part of the host build.
#pragma once

#include <stdint.h>

#include <cmath>
#include <vector>

#include "../../include/vllt.h"
#include "gemm_bf16_epi.cuh"

namespace vllt {

struct SplitKScratch {  // the same fields; the stand-in needs no scratch
  float* part = nullptr;
  int64_t part_bytes = 0;
  int* counters = nullptr;
  int n_counters = 0;
  int max_splits = 0;
};

inline SplitKScratch forward_splitk_scratch(char*) { return SplitKScratch{}; }

template <class Epi>
inline int gemm_bf16_launch(const void* A, int M_cap, const int* M_dev, const void* W, int N, int K, const Epi& epi,
                            int* err, cudaStream_t, const SplitKScratch* = nullptr, int = 0) {
  if (M_cap <= 0 || N <= 0) return VLLT_OK;
  if (K <= 0 || K % 64 != 0 || !err) return VLLT_ERR_ARG;  // the device launcher's checks
  const int M = M_dev ? (*M_dev < M_cap ? *M_dev : M_cap) : M_cap;
  const __nv_bfloat16* a = static_cast<const __nv_bfloat16*>(A);
  const __nv_bfloat16* w = static_cast<const __nv_bfloat16*>(W);
  std::vector<float> arow(K), wt((size_t)32 * K);
  for (int f = 0; f < N; f += 32) {
    for (int j = 0; j < 32; ++j)
      for (int k = 0; k < K; ++k) wt[(size_t)j * K + k] = f + j < N ? __bfloat162float(w[(int64_t)(f + j) * K + k]) : 0.f;
    for (int m = 0; m < M; ++m) {
      for (int k = 0; k < K; ++k) arow[k] = __bfloat162float(a[(int64_t)m * K + k]);
      float v[32];
      for (int j = 0; j < 32; ++j) {
        float acc = 0.f;
        const float* wr = &wt[(size_t)j * K];
        for (int k = 0; k < K; ++k) acc = std::fmaf(arow[k], wr[k], acc);
        v[j] = acc;
      }
      epi.template apply<32>(m, f, v);
    }
  }
  return VLLT_OK;
}

}  // namespace vllt
