// Host side of the tcgen05 bf16 GEMM: tensor maps, launch, C ABI entry.

#include "gemm_bf16_tc.cuh"

using namespace vllt;

extern "C" int vllt_gemm_bf16(const void* A, const void* W, float* C, int32_t M, int32_t N, int32_t K,
                              int32_t* device_flags, void* stream) {
  clear_error();
  VLLT_REQUIRE(M >= 0 && N > 0 && K > 0, "gemm_bf16: bad sizes");
  if (M == 0) return VLLT_OK;
  VLLT_REQUIRE(A && W && C && device_flags, "gemm_bf16: null pointer");
  return gemm_bf16_launch(A, M, nullptr, W, N, K, EpiStoreF32{C, N, N}, device_flags, as_stream(stream));
}
