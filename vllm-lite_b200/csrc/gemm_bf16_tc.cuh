// bf16 GEMM on the 5th-generation tensor cores (tcgen05, TMEM accumulators).
//
//   D[M][N] = A[M][K] . W[N][K]^T      (A and W both K-major bf16, fp32 accumulate)
//
// One CTA (4 warps) computes a 128 x 256 tile:
//   * warp 0 / lane 0 streams A (128 x 64) and W (256 x 64) k-blocks with 2-D TMA
//     loads (128B swizzle) into a 4-stage shared-memory ring (48 KB per stage);
//   * warp 1 / lane 0 issues tcgen05.mma.cta_group::1.kind::f16 (M128 N256 K16, four
//     per k-block) into a 128-lane x 256-column fp32 accumulator in tensor memory and
//     frees each stage with tcgen05.commit on its "empty" mbarrier;
//   * after the last commit all four warps drain the accumulator with
//     tcgen05.ld.32x32b.x32 (warp w owns rows 32w..32w+31) and hand 32 consecutive
//     columns at a time to the epilogue functor.
// No cluster launch and no TMA multicast: the kernel is safe in multi-GPU processes.
// Every mbarrier wait is bounded; on expiry the kernel sets an error bit, lets its
// copies land (bounded), frees its tensor memory and returns.
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace vllt {
namespace tc {

constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4;
constexpr int A_BYTES = BM * BK * 2;            // 16 KB
constexpr int B_BYTES = BN * BK * 2;            // 32 KB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;  // 48 KB
constexpr int TMEM_COLS = 256;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024;  // + alignment slack
constexpr uint64_t kWaitNs = 1000000000ull;

__device__ __forceinline__ uint32_t saddr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(saddr(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(saddr(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, unsigned parity) {
  unsigned ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok) : "r"(saddr(bar)), "r"(parity) : "memory");
  return ok != 0;
}
__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, unsigned parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  while (!mbar_try_wait(bar, parity))
    if (global_ns() - t0 > kWaitNs) return false;
  return true;
}
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(saddr(dst)), "l"(map), "r"(x), "r"(y), "r"(saddr(bar))
      : "memory");
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups 1024 B
// apart (SBO), version 1 (sm_100), base offset 0.
__device__ __forceinline__ uint64_t smem_desc(const void* p) {
  const uint64_t a = (saddr(p) >> 4) & 0x3FFFu;
  return a | (1ull << 16) | (64ull << 32) | (1ull << 46) | (2ull << 61);
}
// Instruction descriptor, kind::f16: fp32 D, bf16 A and B, both K-major, M128 N256.
constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) |
                            ((uint32_t)(BM >> 4) << 24);

__device__ __forceinline__ void mma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n"
      ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(kIdesc), "r"(accumulate));
}
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(saddr(bar))
               : "memory");
}
__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

template <class Epi>
__global__ void __launch_bounds__(128, 1)
gemm_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb, int M_cap,
            const int* __restrict__ M_dev, int N, int K, Epi epi, int* __restrict__ err) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = smem_raw + ((1024 - (saddr(smem_raw) & 1023)) & 1023);
  __shared__ uint64_t full[STAGES], empty[STAGES], accf;
  __shared__ uint32_t tmem_base_s;
  __shared__ int failed_s;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int M = M_dev ? min(*M_dev, M_cap) : M_cap;
  const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
  if (m0 >= M) return;  // uniform over the CTA
  const int nk = K / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(&accf, 1);
    failed_s = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {  // whole warp: allocate the accumulator columns
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(saddr(&tmem_base_s)),
                 "r"(TMEM_COLS));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = tmem_base_s;

  if (warp == 0 && lane == 0) {  // ---- TMA producer ----
    int kb = 0;
    for (; kb < nk; ++kb) {
      const int s = kb % STAGES;
      if (kb >= STAGES && !mbar_wait(&empty[s], ((kb / STAGES) & 1) ^ 1)) {
        atomicOr(err, 4);
        failed_s = 1;
        break;
      }
      unsigned char* a = smem + s * STAGE_BYTES;
      mbar_expect_tx(&full[s], STAGE_BYTES);
      tma_load_2d(a, &ta, &full[s], kb * BK, m0);
      tma_load_2d(a + A_BYTES, &tb, &full[s], kb * BK, n0);
    }
    if (failed_s) {  // let the copies already issued land before the CTA can exit
      for (int j = max(0, kb - STAGES); j < kb; ++j) (void)mbar_wait(&full[j % STAGES], (j / STAGES) & 1);
    }
  } else if (warp == 1 && lane == 0) {  // ---- MMA issuer ----
    bool ok = true;
    for (int kb = 0; kb < nk; ++kb) {
      const int s = kb % STAGES;
      if (!mbar_wait(&full[s], (kb / STAGES) & 1)) {
        atomicOr(err, 4);
        failed_s = 1;
        ok = false;
        break;
      }
      fence_after();
      const unsigned char* a = smem + s * STAGE_BYTES;
      const unsigned char* b = a + A_BYTES;
#pragma unroll
      for (int k = 0; k < BK / 16; ++k)  // +32 bytes per K=16 step inside the swizzled row
        mma_bf16(tmem, smem_desc(a + k * 32), smem_desc(b + k * 32), (kb > 0 || k > 0) ? 1u : 0u);
      mma_commit(&empty[s]);
    }
    if (ok) mma_commit(&accf);
  }
  __syncwarp();

  // ---- epilogue: warp w drains accumulator rows 32w..32w+31 ----
  const bool have = __all_sync(0xffffffffu, mbar_wait(&accf, 0));  // uniform per warp (.aligned loads)
  if (!have && lane == 0) atomicOr(err, 4);
  fence_after();
  if (have) {
    const int row = m0 + warp * 32 + lane;
    const uint32_t lane_addr = tmem + ((uint32_t)(warp * 32) << 16);
#pragma unroll 1
    for (int c = 0; c < BN; c += 32) {
      if (n0 + c >= N) break;  // uniform over the warp
      float v[32];
      tmem_ld32(lane_addr + c, v);
      if (row < M) epi.template apply<32>(row, n0 + c, v);
    }
  }
  fence_before();
  __syncthreads();
  if (warp == 0) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS));
  }
}

}  // namespace tc

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

// ---- host launcher ----------------------------------------------------------------
namespace vllt {

namespace tc {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_fn() {
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
inline int kmajor_map(CUtensorMap* m, const void* base, int64_t rows, int K, int box_rows) {
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

}  // namespace tc

// D = A . W^T through an epilogue. A [M_cap][K], W [N][K] bf16, K % 64 == 0.
template <class Epi>
inline int gemm_bf16_launch(const void* A, int M_cap, const int* M_dev, const void* W, int N, int K, const Epi& epi,
                     int* err, cudaStream_t st) {
  if (M_cap <= 0 || N <= 0) return VLLT_OK;
  VLLT_REQUIRE(K > 0 && K % tc::BK == 0, "gemm_bf16: K must be a positive multiple of 64 (K=%d)", K);
  VLLT_REQUIRE(((uintptr_t)A & 15) == 0 && ((uintptr_t)W & 15) == 0, "gemm_bf16: operands must be 16-byte aligned");
  VLLT_REQUIRE(err, "gemm_bf16: device error word required");
  CUtensorMap ta, tb;
  int rc = tc::kmajor_map(&ta, A, M_cap, K, tc::BM);
  if (rc != VLLT_OK) return rc;
  rc = tc::kmajor_map(&tb, W, N, K, tc::BN);
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

