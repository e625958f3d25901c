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

extern "C" int64_t vllt_gemm_bf16_splitk_workspace_bytes(int32_t M, int32_t N, int32_t K, int32_t splits) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  if (splits <= 0) return align_up(forward_splitk_scratch(nullptr).part_bytes, 256) + align_up(128 * 4, 256);
  const int64_t tiles = (int64_t)ceil_div(N, tc::BN) * ceil_div(M, tc::BM);
  return align_up(splits * tiles * tc::BM * tc::BN * 4, 256) + align_up(tiles * 4, 256);
}

extern "C" int32_t vllt_gemm_bf16_auto_splits(int32_t M, int32_t N, int32_t K) {
  tc::ClusterPlan cp;
  if (cluster_plan(M, N, K, &cp)) return -cp.S;  // cluster split-K form, S CTAs per feature tile
  tc::SmallPlan sp;
  if (small_plan(M, N, K, &sp)) return 0;  // small-M stream-K form
  static char fake;  // non-null stand-in: only the sizes are read
  SplitKScratch sk = forward_splitk_scratch(&fake);
  return choose_splits(M, N, K, &sk);
}

extern "C" int vllt_gemm_bf16_splitk(const void* A, const void* W, float* C, int32_t M, int32_t N, int32_t K,
                                     int32_t splits, void* workspace, int64_t workspace_bytes,
                                     int32_t* device_flags, void* stream) {
  clear_error();
  if (splits < 0) splits = 0;  // the value vllt_gemm_bf16_auto_splits reports for the cluster form
  VLLT_REQUIRE(M >= 0 && N > 0 && K > 0, "gemm_bf16_splitk: bad sizes");
  VLLT_REQUIRE(K % tc::BK == 0 && splits <= K / tc::BK, "gemm_bf16_splitk: splits must be <= K/64 (K=%d)", K);
  if (M == 0) return VLLT_OK;
  VLLT_REQUIRE(A && W && C && device_flags, "gemm_bf16_splitk: null pointer");
  if (splits == 1)
    return gemm_bf16_launch(A, M, nullptr, W, N, K, EpiStoreF32{C, N, N}, device_flags, as_stream(stream), nullptr, 1);
  const int64_t need = vllt_gemm_bf16_splitk_workspace_bytes(M, N, K, splits);
  VLLT_REQUIRE(workspace && workspace_bytes >= need, "gemm_bf16_splitk: workspace %lld < %lld bytes",
               (long long)workspace_bytes, (long long)need);
  SplitKScratch sk;
  if (splits == 0) {  // exactly the forward pass's choice and scratch sizes
    sk = forward_splitk_scratch(reinterpret_cast<char*>(workspace));
  } else {
    const int64_t tiles = (int64_t)ceil_div(N, tc::BN) * ceil_div(M, tc::BM);
    sk.part = reinterpret_cast<float*>(workspace);
    sk.part_bytes = align_up(splits * tiles * tc::BM * tc::BN * 4, 256);
    sk.counters = reinterpret_cast<int*>(reinterpret_cast<char*>(workspace) + sk.part_bytes);
    sk.n_counters = (int)tiles;
    sk.max_splits = splits;
  }
  return gemm_bf16_launch(A, M, nullptr, W, N, K, EpiStoreF32{C, N, N}, device_flags, as_stream(stream), &sk,
                          splits);
}
