// Host side of the tcgen05 bf16 GEMM: tensor maps, launch, C ABI entry.

#include "gemm_bf16_tc.cuh"
#include "ops.cuh"

namespace vllt {

namespace {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(f);
  }
  return fn;
}

// K-major bf16 matrix [rows][K]: boxes of 64 (K) x box_rows, 128-byte swizzle.
int kmajor_map(CUtensorMap* m, const void* base, int64_t rows, int K, int box_rows) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) {
    set_error("gemm_bf16: cuTensorMapEncodeTiled unavailable");
    return VLLT_ERR_CUDA;
  }
  const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)K * 2};
  const cuuint32_t box[2] = {(cuuint32_t)tc::BK, (cuuint32_t)box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("gemm_bf16: cuTensorMapEncodeTiled failed (%d)", (int)r);
    return VLLT_ERR_CUDA;
  }
  return VLLT_OK;
}

}  // namespace

// D = A . W^T through an epilogue. A [M_cap][K], W [N][K] bf16, K % 64 == 0.
template <class Epi>
int gemm_bf16_launch(const void* A, int M_cap, const int* M_dev, const void* W, int N, int K, const Epi& epi,
                     int* err, cudaStream_t st) {
  if (M_cap <= 0 || N <= 0) return VLLT_OK;
  VLLT_REQUIRE(K > 0 && K % tc::BK == 0, "gemm_bf16: K must be a positive multiple of 64 (K=%d)", K);
  VLLT_REQUIRE(((uintptr_t)A & 15) == 0 && ((uintptr_t)W & 15) == 0, "gemm_bf16: operands must be 16-byte aligned");
  VLLT_REQUIRE(err, "gemm_bf16: device error word required");
  CUtensorMap ta, tb;
  int rc = kmajor_map(&ta, A, M_cap, K, tc::BM);
  if (rc != VLLT_OK) return rc;
  rc = kmajor_map(&tb, W, N, K, tc::BN);
  if (rc != VLLT_OK) return rc;
  static unsigned configured = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 32 && !(configured & (1u << dev))) {
    cudaFuncSetAttribute(tc::gemm_kernel<Epi>, cudaFuncAttributeMaxDynamicSharedMemorySize, tc::SMEM_BYTES);
    configured |= 1u << dev;
  }
  dim3 grid(ceil_div(N, tc::BN), ceil_div(M_cap, tc::BM));
  tc::gemm_kernel<Epi><<<grid, 128, tc::SMEM_BYTES, st>>>(ta, tb, M_cap, M_dev, N, K, epi, err);
  return check_launch("gemm_bf16");
}

}  // namespace vllt

using namespace vllt;

extern "C" int vllt_gemm_bf16(const void* A, const void* W, float* C, int32_t M, int32_t N, int32_t K,
                              int32_t* device_flags, void* stream) {
  clear_error();
  VLLT_REQUIRE(M >= 0 && N > 0 && K > 0, "gemm_bf16: bad sizes");
  if (M == 0) return VLLT_OK;
  VLLT_REQUIRE(A && W && C && device_flags, "gemm_bf16: null pointer");
  return gemm_bf16_launch(A, M, nullptr, W, N, K, EpiStoreF32{C, N, N}, device_flags, as_stream(stream));
}
