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
// Two forms share this pipeline:
//   * gemm_persistent_kernel (unsplit): one CTA per SM walks the tiles in a
//     grouped raster; 6 warps (TMA, MMA, 4 epilogue) and two TMEM accumulators,
//     so a tile's epilogue overlaps the next tile's main loop;
//   * gemm_kernel with split-K (gridDim.z > 1, for the small-M decode passes
//     whose tile grid would leave most SMs idle): CTA z accumulates k-blocks
//     [z*nk/s, (z+1)*nk/s), stores its fp32 tile to a partials buffer, and the
//     last CTA of each tile to arrive (per-tile counter) sums the partials in z
//     order, so the result does not depend on arrival order, applies the
//     epilogue and resets the counter.
// No TMA multicast anywhere (the cluster form shares data through distributed
// shared memory only): the kernels are safe in multi-GPU processes.
// Every mbarrier wait is bounded; on expiry the kernel sets an error bit, lets its
// copies land (bounded), frees its tensor memory and returns.
// Under the host emulation (VLLT_SIMT_HOST, tests/simt_host.h) the helpers
// written in inline PTX are the emulation's tensor-core, TMA, mbarrier and
// cluster operations (tests/simt_include/simt_tc.h), so the CPU tests run
// these kernels' own code.
#pragma once

#include <cuda.h>

#include <algorithm>

#include "common.cuh"
#ifdef VLLT_SIMT_HOST
#include <simt_tc.h>
#endif

namespace vllt {
namespace tc {

constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4;
constexpr int GROUP_M = 16;  // row tiles per raster group
constexpr int A_BYTES = BM * BK * 2;            // 16 KB
constexpr int B_BYTES = BN * BK * 2;            // 32 KB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;  // 48 KB
constexpr int TMEM_COLS = 256;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024;  // + alignment slack
constexpr uint64_t kWaitNs = 1000000000ull;

#ifdef VLLT_SIMT_HOST
inline uint32_t saddr(const void* p) { return ::simt::tensor::saddr(p); }
inline void mbar_init(uint64_t* bar, unsigned count) { ::simt::tensor::mbar_init(bar, count); }
inline void mbar_expect_tx(uint64_t* bar, unsigned bytes) { ::simt::tensor::mbar_expect_tx(bar, bytes); }
inline bool mbar_try_wait(uint64_t* bar, unsigned parity) { return ::simt::tensor::mbar_try_wait(bar, parity); }
inline uint64_t global_ns() { return ::simt::tensor::global_ns(); }
inline void mbar_arrive(uint64_t* bar) { ::simt::tensor::mbar_arrive(bar); }
inline void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  ::simt::tensor::tma_load(dst, map, bar, x, y, 0);
}
inline void mma_commit(uint64_t* bar) { ::simt::tensor::mma_commit(bar); }
inline void fence_before() {}
inline void fence_after() {}
inline void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  ::simt::tensor::tmem_ld32(taddr, r);
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
inline void mbar_fence_init() {}
inline void tmem_alloc(uint32_t* dst, uint32_t ncols) { ::simt::tensor::tmem_alloc(dst, ncols); }
inline void tmem_relinquish() { ::simt::tensor::tmem_relinquish(); }
inline void tmem_dealloc(uint32_t taddr, uint32_t ncols) { ::simt::tensor::tmem_dealloc(taddr, ncols); }
#else
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
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(saddr(bar)) : "memory");
}
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(saddr(dst)), "l"(map), "r"(x), "r"(y), "r"(saddr(bar))
      : "memory");
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
__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
// The warp allocates `ncols` columns of tensor memory; their address goes to *dst.
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(saddr(dst)), "r"(ncols));
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols));
}
#endif
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, unsigned parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  while (!mbar_try_wait(bar, parity))
    if (global_ns() - t0 > kWaitNs) return false;
  return true;
}
// The abort flag one role of a CTA raises and the other roles poll while they
// wait: a volatile shared-memory word on the device (relaxed accesses in the
// PTX memory model), a relaxed atomic under the host emulation, where the
// roles run as concurrent threads that the race check watches.
__device__ __forceinline__ int flag_read(const volatile int* f) {
#ifdef VLLT_SIMT_HOST
  return __atomic_load_n(const_cast<const int*>(f), __ATOMIC_RELAXED);
#else
  return *f;
#endif
}
__device__ __forceinline__ void flag_write(volatile int* f, int v) {
#ifdef VLLT_SIMT_HOST
  __atomic_store_n(const_cast<int*>(f), v, __ATOMIC_RELAXED);
#else
  *f = v;
#endif
}
// As mbar_wait, but also gives up as soon as another role of the CTA has set *abort.
__device__ __forceinline__ bool mbar_wait_or_abort(uint64_t* bar, unsigned parity, volatile int* abort) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (flag_read(abort)) return false;
    if (global_ns() - t0 > kWaitNs) return false;
  }
  return true;
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

#ifdef VLLT_SIMT_HOST
inline void mma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
  ::simt::tensor::mma_f16(tmem_d, adesc, bdesc, kIdesc, accumulate);
}
#else
__device__ __forceinline__ void mma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n"
      ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(kIdesc), "r"(accumulate));
}
#endif

// Grouped raster order of output tiles (both kernels): consecutive tile ids
// walk up to GROUP_M row tiles of one column tile, then the next column tile,
// so the CTAs resident at one time share a few A row slabs and W column slabs
// in L2 instead of streaming all of W once per row slab.
__device__ __forceinline__ void tile_origin(int t, int n_tiles, int m_tiles, int& m0, int& n0) {
  const int per_group = GROUP_M * n_tiles;
  const int first_m = (t / per_group) * GROUP_M, gm = min(m_tiles - first_m, GROUP_M);
  const int r = t % per_group;
  m0 = (first_m + r % gm) * BM;
  n0 = (r / gm) * BN;
}

struct SplitK {
  float* part;    // [splits][tiles][BM][BN] fp32 partial tiles
  int* counters;  // [tiles], zero between launches
};

template <class Epi>
__global__ void __launch_bounds__(128, 1)
gemm_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb, int M_cap,
            const int* __restrict__ M_dev, int N, int K, Epi epi, int* __restrict__ err, SplitK sk) {
  VLLT_DYNAMIC_SMEM(smem_raw, 1024);
  unsigned char* smem = smem_raw + ((1024 - (saddr(smem_raw) & 1023)) & 1023);
  __shared__ uint64_t full[STAGES], empty[STAGES], accf;
  __shared__ uint32_t tmem_base_s;
  __shared__ int last_s;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int M = M_dev ? min(*M_dev, M_cap) : M_cap;
  const int n_tiles = (N + BN - 1) / BN;
  int m0, n0;
  tile_origin(blockIdx.x, n_tiles, gridDim.x / n_tiles, m0, n0);
  if (m0 >= M) return;  // uniform over the CTA (and over every split of this tile)
  const int splits = gridDim.z;
  const int kb0 = (int)((int64_t)blockIdx.z * (K / BK) / splits);
  const int nk = (int)((int64_t)(blockIdx.z + 1) * (K / BK) / splits) - kb0;  // >= 1 (host: splits <= K/BK)

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(&accf, 1);
    mbar_fence_init();
  }
  if (warp == 0) {  // whole warp: allocate the accumulator columns
    tmem_alloc(&tmem_base_s, TMEM_COLS);
    tmem_relinquish();
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
        break;
      }
      unsigned char* a = smem + s * STAGE_BYTES;
      mbar_expect_tx(&full[s], STAGE_BYTES);
      tma_load_2d(a, &ta, &full[s], (kb0 + kb) * BK, m0);
      tma_load_2d(a + A_BYTES, &tb, &full[s], (kb0 + kb) * BK, n0);
    }
    // The copies issued last land before the CTA can exit, whichever role gave
    // up (immediate when nothing failed: the epilogue waits for them anyway).
    for (int j = max(0, kb - STAGES); j < kb; ++j) (void)mbar_wait(&full[j % STAGES], (j / STAGES) & 1);
  } else if (warp == 1 && lane == 0) {  // ---- MMA issuer ----
    bool ok = true;
    for (int kb = 0; kb < nk; ++kb) {
      const int s = kb % STAGES;
      if (!mbar_wait(&full[s], (kb / STAGES) & 1)) {
        atomicOr(err, 4);
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
  const int row = m0 + warp * 32 + lane;
  const uint32_t lane_addr = tmem + ((uint32_t)(warp * 32) << 16);
  if (splits == 1) {
    if (have) {
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        if (n0 + c >= N) break;  // uniform over the warp
        float v[32];
        tmem_ld32(lane_addr + c, v);
        if (row < M) epi.template apply<32>(row, n0 + c, v);
      }
    }
  } else {
    const int tiles = gridDim.x, tile = blockIdx.x;
    const int64_t zstride = (int64_t)tiles * BM * BN;
    float* mine = sk.part + (int64_t)tile * BM * BN + (int64_t)(warp * 32 + lane) * BN;
    if (have) {
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        if (n0 + c >= N) break;
        float v[32];
        tmem_ld32(lane_addr + c, v);
        float4* dst = reinterpret_cast<float4*>(mine + blockIdx.z * zstride + c);
#pragma unroll
        for (int j = 0; j < 8; ++j) __stcg(dst + j, make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]));
      }
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) last_s = atomicAdd(&sk.counters[tile], 1) == splits - 1;
    __syncthreads();
    if (last_s) {  // every split has stored its tile: sum them in z order
      __threadfence();
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        if (n0 + c >= N) break;
        float v[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = 0.f;
#pragma unroll 1
        for (int z = 0; z < splits; ++z) {
          const float4* src = reinterpret_cast<const float4*>(mine + z * zstride + c);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float4 t = __ldcg(src + j);
            v[4 * j] += t.x; v[4 * j + 1] += t.y; v[4 * j + 2] += t.z; v[4 * j + 3] += t.w;
          }
        }
        if (row < M) epi.template apply<32>(row, n0 + c, v);
      }
      if (threadIdx.x == 0) sk.counters[tile] = 0;  // ready for the next launch on this stream
    }
  }
  fence_before();
  __syncthreads();
  if (warp == 0) {
    fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

// Persistent, warp-specialized form for the unsplit case: one CTA per SM walks
// tiles blockIdx.x, blockIdx.x + gridDim.x, ... Warp 0 streams k-blocks through
// the shared-memory ring without pausing between tiles, warp 1 issues the MMAs
// into one of two 256-column TMEM accumulators (512 columns), and warps 2-5
// drain the other accumulator through the epilogue at the same time.
constexpr int P_THREADS = 192;
constexpr int P_TMEM_COLS = 512;

template <class Epi>
__global__ void __launch_bounds__(P_THREADS, 1)
gemm_persistent_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb, int M_cap,
                       const int* __restrict__ M_dev, int N, int K, Epi epi, int* __restrict__ err) {
  VLLT_DYNAMIC_SMEM(smem_raw, 1024);
  unsigned char* smem = smem_raw + ((1024 - (saddr(smem_raw) & 1023)) & 1023);
  __shared__ uint64_t full[STAGES], empty[STAGES], acc_full[2], acc_empty[2], drain;
  __shared__ uint32_t tmem_base_s;
  __shared__ volatile int abort_s;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int M = M_dev ? min(*M_dev, M_cap) : M_cap;
  const int n_tiles = (N + BN - 1) / BN, m_tiles = (M + BM - 1) / BM;
  const int total = n_tiles * m_tiles, nk = K / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 4);  // one arrival per epilogue warp
    }
    mbar_init(&drain, 1);
    flag_write(&abort_s, 0);
    mbar_fence_init();
  }
  if (warp == 0) {
    tmem_alloc(&tmem_base_s, P_TMEM_COLS);
    tmem_relinquish();
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = tmem_base_s;

  if (warp == 0) {
    if (lane == 0) {  // ---- TMA producer ----
      int g = 0;
      bool failed = false;
      for (int t = blockIdx.x; t < total && !failed; t += gridDim.x) {
        int m0, n0;
        tile_origin(t, n_tiles, m_tiles, m0, n0);
        for (int kb = 0; kb < nk; ++kb, ++g) {
          const int s = g % STAGES;
          if (g >= STAGES && !mbar_wait_or_abort(&empty[s], ((g / STAGES) & 1) ^ 1, &abort_s)) {
            failed = true;
            break;
          }
          unsigned char* a = smem + s * STAGE_BYTES;
          mbar_expect_tx(&full[s], STAGE_BYTES);
          tma_load_2d(a, &ta, &full[s], kb * BK, m0);
          tma_load_2d(a + A_BYTES, &tb, &full[s], kb * BK, n0);
        }
      }
      if (failed) {
        atomicOr(err, 4);
        flag_write(&abort_s, 1);
        // let the copies already issued land before the CTA can exit
        for (int j = max(0, g - STAGES); j < g; ++j) (void)mbar_wait(&full[j % STAGES], (j / STAGES) & 1);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {  // ---- MMA issuer ----
      int g = 0, i = 0;
      bool failed = false;
      for (int t = blockIdx.x; t < total && !failed; t += gridDim.x, ++i) {
        const int a = i & 1;
        if (i >= 2 && !mbar_wait_or_abort(&acc_empty[a], ((i >> 1) & 1) ^ 1, &abort_s)) {
          failed = true;
          break;
        }
        fence_after();
        const uint32_t d = tmem + a * BN;
        for (int kb = 0; kb < nk; ++kb, ++g) {
          const int s = g % STAGES;
          if (!mbar_wait_or_abort(&full[s], (g / STAGES) & 1, &abort_s)) {
            failed = true;
            break;
          }
          fence_after();
          const unsigned char* sa = smem + s * STAGE_BYTES;
          const unsigned char* sb = sa + A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            mma_bf16(d, smem_desc(sa + k * 32), smem_desc(sb + k * 32), (kb > 0 || k > 0) ? 1u : 0u);
          mma_commit(&empty[s]);
        }
        if (!failed) mma_commit(&acc_full[a]);
      }
      if (failed) {
        atomicOr(err, 4);
        flag_write(&abort_s, 1);
      }
      if (g > 0) {  // every MMA this thread issued has finished before the columns are freed
        mma_commit(&drain);
        (void)mbar_wait(&drain, 0);
      }
    }
  } else {  // ---- epilogue warps 2..5: TMEM lane quarter (warp % 4) ----
    const int q = warp & 3;
    int i = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x, ++i) {
      const int a = i & 1;
      const bool have = __all_sync(0xffffffffu, mbar_wait_or_abort(&acc_full[a], (i >> 1) & 1, &abort_s));
      if (!have) {
        if (lane == 0) {
          atomicOr(err, 4);
          flag_write(&abort_s, 1);
        }
        break;
      }
      fence_after();
      int m0, n0;
      tile_origin(t, n_tiles, m_tiles, m0, n0);
      const int row = m0 + q * 32 + lane;
      const uint32_t lane_addr = tmem + a * BN + ((uint32_t)(q * 32) << 16);
#pragma unroll 1
      for (int c = 0; c < BN; c += 32) {
        if (n0 + c >= N) break;  // uniform over the warp
        float v[32];
        tmem_ld32(lane_addr + c, v);
        if (row < M) epi.template apply<32>(row, n0 + c, v);
      }
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[a]);
    }
  }
  fence_before();
  __syncthreads();
  if (warp == 0) {
    fence_after();
    tmem_dealloc(tmem, P_TMEM_COLS);
  }
}

// ---- small-M form (decode passes): weights on the MMA's M side -----------------------
//
// With few token rows (M <= 256) a 128-row token tile wastes most of the
// tensor core and the tile grid covers few SMs, while the run time is set by
// streaming W once from HBM. This form swaps the operands: the MMA computes
// D^T[128 features][n_pad tokens] = W_tile . A^T (both K-major in shared
// memory, M128 x N n_pad x K16), so one CTA covers 128 output features for
// every token. Work is cut stream-K: the (feature tile, k-block) iterations
// are divided evenly over one CTA per SM, so every SM streams the same number
// of weight bytes whatever the shape. A CTA's span covers whole tiles, whose
// epilogue it applies itself (transposed through shared memory so the
// epilogue sees 32 consecutive features of one token), and at most two partial
// tiles at its ends, which it stores as fp32 [token][128] slices; a second
// kernel sums each split tile's slices in CTA order (deterministic) and
// applies the epilogue.
constexpr int SK_THREADS = 192;             // warps 0-3 epilogue, warp 4 TMA, warp 5 MMA
constexpr int SK_W_BYTES = 128 * BK * 2;    // one 128-feature x 64 k weight tile (16 KB)
constexpr int SK_MAX_STAGES = 8;
constexpr int SK_RING_BYTES = 192 * 1024;
constexpr int SK_TBUF_BYTES = 4 * 32 * 33 * 4;  // per-warp 32 x 33 transpose buffers

struct SmallPlan {
  int tiles;      // ceil(N / 128)
  int ksub;       // 64-wide k sub-blocks per iteration (longer contiguous weight rows per load)
  int nk;         // K / (64 * ksub)
  int ctas;       // CTAs; CTA c owns iterations [c*total/ctas, (c+1)*total/ctas)
  int n_pad;      // MMA N (tokens, padded: 32..256, power of two)
  int stages;
  int64_t total;  // tiles * nk
};

__device__ __forceinline__ int64_t sk_begin(int c, const SmallPlan& p) { return (int64_t)c * p.total / p.ctas; }
__device__ __forceinline__ int sk_owner(int64_t it, const SmallPlan& p) {
  return (int)(((it + 1) * p.ctas - 1) / p.total);
}
// slot of CTA c's partial slice of tile t: 2c for its first tile, 2c+1 for its last
__device__ __forceinline__ int sk_slot(int c, int t, const SmallPlan& p) {
  return 2 * c + (t == (int)(sk_begin(c, p) / p.nk) ? 0 : 1);
}

#ifdef VLLT_SIMT_HOST
inline void mma_bf16_n(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  ::simt::tensor::mma_f16(tmem_d, adesc, bdesc, idesc, accumulate);
}
#else
__device__ __forceinline__ void mma_bf16_n(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n"
      ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}
#endif

template <class Epi>
__global__ void __launch_bounds__(SK_THREADS, 1)
gemm_small_kernel(const __grid_constant__ CUtensorMap tw, const __grid_constant__ CUtensorMap tx, int M_cap,
                  const int* __restrict__ M_dev, int N, SmallPlan p, Epi epi, float* __restrict__ part,
                  int* __restrict__ err) {
  VLLT_DYNAMIC_SMEM(smem_raw, 1024);
  unsigned char* smem = smem_raw + ((1024 - (saddr(smem_raw) & 1023)) & 1023);
  __shared__ uint64_t full[SK_MAX_STAGES], empty[SK_MAX_STAGES], acc_full[2], acc_empty[2], drain;
  __shared__ uint32_t tmem_base_s;
  __shared__ volatile int abort_s;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int stages = p.stages, nk = p.nk, ksub = p.ksub;
  const uint32_t x_bytes = (uint32_t)p.n_pad * 128;  // one 64-wide k sub-block of the token tile
  const uint32_t stage_bytes = ksub * (SK_W_BYTES + x_bytes);  // [W sub-blocks][token sub-blocks]
  float* tbuf = reinterpret_cast<float*>(smem + stages * stage_bytes);
  const int64_t it_begin = sk_begin(blockIdx.x, p), it_end = sk_begin(blockIdx.x + 1, p);
  const uint32_t tmem_cols = 2 * p.n_pad;  // two accumulators (64..512, a power of two)
  const uint32_t idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(p.n_pad >> 3) << 17) |
                         ((uint32_t)(128 >> 4) << 24);

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 4);
    }
    mbar_init(&drain, 1);
    flag_write(&abort_s, 0);
    mbar_fence_init();
  }
  if (warp == 0) {
    tmem_alloc(&tmem_base_s, tmem_cols);
    tmem_relinquish();
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = tmem_base_s;
  // weights do not depend on earlier kernels: the first ring slots' W tiles
  // are requested before waiting for the previous kernel (launched with PDL)
  const int pre = (int)min((int64_t)stages, it_end - it_begin);
  if (warp == 4 && lane == 0) {
    for (int g = 0; g < pre; ++g) {
      const int64_t it = it_begin + g;
      mbar_expect_tx(&full[g], stage_bytes);
      for (int u = 0; u < ksub; ++u)
        tma_load_2d(smem + g * stage_bytes + u * SK_W_BYTES, &tw, &full[g], ((int)(it % nk) * ksub + u) * BK,
                    (int)(it / nk) * 128);
    }
  }
  pdl_wait();  // (no early trigger: the reduce kernel's CTAs parked beside this one slow it down)
  const int M = M_dev ? min(*M_dev, M_cap) : M_cap;  // 0 rows: the pipeline runs, nothing is stored

  if (warp == 4) {
    if (lane == 0) {  // ---- TMA producer: W tile and the token tile of each k-block ----
      int g = 0;
      bool failed = false;
      for (int64_t it = it_begin; it < it_end; ++it, ++g) {
        const int t = (int)(it / nk), kb = (int)(it % nk);
        const int s = g % stages;
        unsigned char* a = smem + s * stage_bytes;
        unsigned char* ax = a + ksub * SK_W_BYTES;
        if (g >= pre) {  // else W was requested before the PDL wait
          if (!mbar_wait_or_abort(&empty[s], ((g / stages) & 1) ^ 1, &abort_s)) {
            failed = true;
            break;
          }
          mbar_expect_tx(&full[s], stage_bytes);
          for (int u = 0; u < ksub; ++u) tma_load_2d(a + u * SK_W_BYTES, &tw, &full[s], (kb * ksub + u) * BK, t * 128);
        }
        for (int u = 0; u < ksub; ++u) tma_load_2d(ax + u * x_bytes, &tx, &full[s], (kb * ksub + u) * BK, 0);
      }
      if (failed) {
        atomicOr(err, 4);
        flag_write(&abort_s, 1);
        for (int j = max(0, g - stages); j < g; ++j) (void)mbar_wait(&full[j % stages], (j / stages) & 1);
      }
    }
  } else if (warp == 5) {
    if (lane == 0) {  // ---- MMA issuer: one accumulator per tile segment, alternating ----
      int g = 0, seg = 0;
      bool failed = false;
      int64_t it = it_begin;
      while (it < it_end && !failed) {
        const int t = (int)(it / nk);
        const int64_t seg_begin = it, seg_end = min(it_end, (int64_t)(t + 1) * nk);
        const int a = seg & 1;
        if (seg >= 2 && !mbar_wait_or_abort(&acc_empty[a], ((seg >> 1) & 1) ^ 1, &abort_s)) {
          failed = true;
          break;
        }
        fence_after();
        const uint32_t d = tmem + a * p.n_pad;
        for (; it < seg_end; ++it, ++g) {
          const int s = g % stages;
          if (!mbar_wait_or_abort(&full[s], (g / stages) & 1, &abort_s)) {
            failed = true;
            break;
          }
          fence_after();
          const unsigned char* sw0 = smem + s * stage_bytes;
          const unsigned char* sx0 = sw0 + ksub * SK_W_BYTES;
          for (int u = 0; u < ksub; ++u) {
            const unsigned char* sw = sw0 + u * SK_W_BYTES;
            const unsigned char* sx = sx0 + u * x_bytes;
#pragma unroll
            for (int k = 0; k < BK / 16; ++k)
              mma_bf16_n(d, smem_desc(sw + k * 32), smem_desc(sx + k * 32), idesc,
                         (it > seg_begin || u > 0 || k > 0) ? 1u : 0u);
          }
          mma_commit(&empty[s]);
        }
        if (!failed) mma_commit(&acc_full[a]);
        ++seg;
      }
      if (failed) {
        atomicOr(err, 4);
        flag_write(&abort_s, 1);
      }
      if (g > 0) {
        mma_commit(&drain);
        (void)mbar_wait(&drain, 0);
      }
    }
  } else {  // ---- epilogue warps 0-3: features 32*warp .. +31 of the tile (TMEM lanes) ----
    float* tb = tbuf + warp * 32 * 33;
    int seg = 0;
    int64_t it = it_begin;
    const int t_first = (int)(it_begin / nk);
    while (it < it_end) {
      const int t = (int)(it / nk);
      const int64_t seg_end = min(it_end, (int64_t)(t + 1) * nk);
      const bool whole = (it == (int64_t)t * nk) && (seg_end == (int64_t)(t + 1) * nk);
      const int a = seg & 1;
      const bool have = __all_sync(0xffffffffu, mbar_wait_or_abort(&acc_full[a], (seg >> 1) & 1, &abort_s));
      if (!have) {
        if (lane == 0) {
          atomicOr(err, 4);
          flag_write(&abort_s, 1);
        }
        break;
      }
      fence_after();
      const int f0 = t * 128 + warp * 32;
      const uint32_t lane_addr = tmem + a * p.n_pad + ((uint32_t)(warp * 32) << 16);
      float* slice = whole ? nullptr
                           : part + (int64_t)(2 * blockIdx.x + (t == t_first ? 0 : 1)) * M_cap * 128 + warp * 32 + lane;
#pragma unroll 1
      for (int c = 0; c < p.n_pad; c += 32) {
        if (c >= M || f0 >= N) break;  // uniform over the warp
        float v[32];
        tmem_ld32(lane_addr + c, v);  // v[j] = D^T[feature f0 + lane][token c + j]
        if (!whole) {                 // fp32 slice [token][128]: 32 consecutive floats per store
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (c + j < M) __stcg(slice + (int64_t)(c + j) * 128, v[j]);
          continue;
        }
#pragma unroll
        for (int j = 0; j < 32; ++j) tb[lane * 33 + j] = v[j];
        __syncwarp();
        float u[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) u[i] = tb[i * 33 + lane];  // token c + lane, features f0 + i
        __syncwarp();
        if (c + lane < M) epi.template apply<32>(c + lane, f0, u);
      }
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[a]);
      it = seg_end;
      ++seg;
    }
  }
  fence_before();
  __syncthreads();
  if (warp == 0) {
    fence_after();
    tmem_dealloc(tmem, tmem_cols);
  }
}

// ---- small-M form with few feature tiles: split-K inside a thread-block cluster ----
//
// When N / 128 feature tiles cannot cover the SMs, the S CTAs of a cluster
// share one tile: CTA r (cluster rank) accumulates k-blocks [r*nk/S,
// (r+1)*nk/S) in TMEM, stages the fp32 accumulator in its own shared memory as
// [token][128 features], and after a cluster barrier sums token rows
// [r*n/S, (r+1)*n/S) over the S CTAs' buffers (distributed shared memory,
// rank order: deterministic) and applies the epilogue. No partials go through
// global memory and no second kernel runs. The ring is reused for the staging
// buffer once the last MMA has completed.
// A location in another CTA's shared memory: its shared::cluster address on the
// device, a pointer under the host emulation; `+ bytes` moves along it.
#ifdef VLLT_SIMT_HOST
typedef const unsigned char* PeerAddr;
inline uint32_t cluster_rank() { return ::simt::tensor::cluster_rank(); }
inline void cluster_sync() { ::simt::tensor::cluster_sync(); }
inline PeerAddr peer_addr(const void* p, uint32_t rank) {
  return static_cast<PeerAddr>(::simt::map_shared(p, (int)rank));
}
inline int ld_peer_s32(PeerAddr a) {
  int v;
  memcpy(&v, a, 4);
  return v;
}
inline float4 ld_peer4(PeerAddr a) {
  float4 v;
  memcpy(&v, a, 16);
  return v;
}
#else
typedef uint32_t PeerAddr;
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// p (this CTA's shared memory) -> the same offset in CTA `rank` of the cluster
__device__ __forceinline__ PeerAddr peer_addr(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr(p)), "r"(rank));
  return r;
}
__device__ __forceinline__ int ld_peer_s32(PeerAddr addr) {
  int v;
  asm volatile("ld.shared::cluster.s32 %0, [%1];" : "=r"(v) : "r"(addr) : "memory");
  return v;
}
__device__ __forceinline__ float4 ld_peer4(PeerAddr addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr) : "memory");
  return v;
}
#endif

struct ClusterPlan {
  int tiles;   // ceil(N / 128)
  int S;       // CTAs per tile = cluster size
  int ksub, nk;  // k sub-blocks per stage; iterations of the whole K
  int n_pad, stages;
};

template <class Epi>
__global__ void __launch_bounds__(SK_THREADS, 1)
gemm_cluster_kernel(const __grid_constant__ CUtensorMap tw, const __grid_constant__ CUtensorMap tx, int M_cap,
                    const int* __restrict__ M_dev, int N, ClusterPlan p, Epi epi, int* __restrict__ err) {
  VLLT_DYNAMIC_SMEM(smem_raw, 1024);
  unsigned char* smem = smem_raw + ((1024 - (saddr(smem_raw) & 1023)) & 1023);
  __shared__ uint64_t full[SK_MAX_STAGES], empty[SK_MAX_STAGES], acc_full, drain;
  __shared__ uint32_t tmem_base_s;
  __shared__ volatile int abort_s;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int stages = p.stages, ksub = p.ksub;
  const uint32_t x_bytes = (uint32_t)p.n_pad * 128;
  const uint32_t stage_bytes = ksub * (SK_W_BYTES + x_bytes);
  const int rank = (int)cluster_rank();
  const int t = blockIdx.x / p.S;
  const int kb0 = rank * p.nk / p.S, kb1 = (rank + 1) * p.nk / p.S, n_it = kb1 - kb0;
  const uint32_t tmem_cols = p.n_pad < 32 ? 32 : p.n_pad;
  const uint32_t idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(p.n_pad >> 3) << 17) |
                         ((uint32_t)(128 >> 4) << 24);
  float* stage_acc = reinterpret_cast<float*>(smem);  // [n_pad tokens][128 features], after the main loop

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(&acc_full, 1);
    mbar_init(&drain, 1);
    flag_write(&abort_s, 0);
    mbar_fence_init();
  }
  if (warp == 0) {
    tmem_alloc(&tmem_base_s, tmem_cols);
    tmem_relinquish();
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = tmem_base_s;
  const int pre = min(stages, n_it);
  if (warp == 4 && lane == 0) {  // weights first: they do not depend on the previous kernel
    for (int g = 0; g < pre; ++g) {
      mbar_expect_tx(&full[g], stage_bytes);
      for (int u = 0; u < ksub; ++u)
        tma_load_2d(smem + g * stage_bytes + u * SK_W_BYTES, &tw, &full[g], ((kb0 + g) * ksub + u) * BK, t * 128);
    }
  }
  pdl_wait();
  const int M = M_dev ? min(*M_dev, M_cap) : M_cap;

  if (warp == 4) {
    if (lane == 0) {  // ---- TMA producer ----
      int g = 0;
      bool failed = false;
      for (; g < n_it; ++g) {
        const int s = g % stages, kb = kb0 + g;
        unsigned char* a = smem + s * stage_bytes;
        unsigned char* ax = a + ksub * SK_W_BYTES;
        if (g >= pre) {
          if (!mbar_wait_or_abort(&empty[s], ((g / stages) & 1) ^ 1, &abort_s)) {
            failed = true;
            break;
          }
          mbar_expect_tx(&full[s], stage_bytes);
          for (int u = 0; u < ksub; ++u) tma_load_2d(a + u * SK_W_BYTES, &tw, &full[s], (kb * ksub + u) * BK, t * 128);
        }
        for (int u = 0; u < ksub; ++u) tma_load_2d(ax + u * x_bytes, &tx, &full[s], (kb * ksub + u) * BK, 0);
      }
      if (failed) {
        atomicOr(err, 4);
        flag_write(&abort_s, 1);
        for (int j = max(0, g - stages); j < g; ++j) (void)mbar_wait(&full[j % stages], (j / stages) & 1);
      }
    }
  } else if (warp == 5) {
    if (lane == 0) {  // ---- MMA issuer ----
      int g = 0;
      bool failed = false;
      for (; g < n_it; ++g) {
        const int s = g % stages;
        if (!mbar_wait_or_abort(&full[s], (g / stages) & 1, &abort_s)) {
          failed = true;
          break;
        }
        fence_after();
        const unsigned char* sw0 = smem + s * stage_bytes;
        const unsigned char* sx0 = sw0 + ksub * SK_W_BYTES;
        for (int u = 0; u < ksub; ++u) {
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            mma_bf16_n(tmem, smem_desc(sw0 + u * SK_W_BYTES + k * 32), smem_desc(sx0 + u * x_bytes + k * 32), idesc,
                       (g > 0 || u > 0 || k > 0) ? 1u : 0u);
        }
        mma_commit(&empty[s]);
      }
      if (!failed && n_it > 0) mma_commit(&acc_full);
      if (failed) {
        atomicOr(err, 4);
        flag_write(&abort_s, 1);
      }
      if (g > 0) {
        mma_commit(&drain);
        (void)mbar_wait(&drain, 0);
      }
    }
  } else {  // ---- epilogue warps 0-3: TMEM lanes = features 32*warp .. +31 -> staging buffer ----
    const bool have = __all_sync(0xffffffffu, mbar_wait_or_abort(&acc_full, 0, &abort_s));
    if (!have) {
      if (lane == 0) {
        atomicOr(err, 4);
        flag_write(&abort_s, 1);
      }
    } else {
      fence_after();
      const uint32_t lane_addr = tmem + ((uint32_t)(warp * 32) << 16);
#pragma unroll 1
      for (int c = 0; c < p.n_pad; c += 32) {
        if (c >= M) break;
        float v[32];
        tmem_ld32(lane_addr + c, v);  // v[j] = D^T[feature 32*warp + lane][token c + j]
#pragma unroll
        for (int j = 0; j < 32; ++j) stage_acc[(c + j) * 128 + warp * 32 + lane] = v[j];
      }
    }
  }
  // every CTA of the cluster has staged its accumulator (or failed; the error bit is set)
  __syncthreads();
  __syncwarp();
  cluster_sync();
  // A CTA that gave up never wrote its staging buffer: then no CTA of the
  // cluster reduces or runs the epilogue (which may write the KV cache). Each
  // CTA set its own abort_s before the barrier above (release / acquire), so
  // the peers' values read here are final.
  bool cluster_ok = !flag_read(&abort_s);
  if (warp < 4)
    for (int src = 0; src < p.S && cluster_ok; ++src)
      cluster_ok = ld_peer_s32(peer_addr(const_cast<int*>(&abort_s), src)) == 0;
  if (warp < 4 && cluster_ok) {  // ---- reduction of token rows [r*n/S, (r+1)*n/S) ----
    const int n_tok = min(M, p.n_pad);
    const int r0 = rank * n_tok / p.S, r1 = (rank + 1) * n_tok / p.S;
    for (int item = threadIdx.x; item < (r1 - r0) * 4; item += 128) {
      const int m = r0 + item / 4, q = item % 4;
      const int f = t * 128 + q * 32;
      if (f >= N) continue;
      float v[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = 0.f;
      for (int src = 0; src < p.S; ++src) {
        const PeerAddr ra = peer_addr(stage_acc + m * 128 + q * 32, src);
        float4 r[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) r[j] = ld_peer4(ra + j * 16);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          v[4 * j] += r[j].x; v[4 * j + 1] += r[j].y; v[4 * j + 2] += r[j].z; v[4 * j + 3] += r[j].w;
        }
      }
      epi.template apply<32>(m, f, v);
    }
  }
  __syncwarp();
  cluster_sync();  // no CTA leaves while another still reads its buffer
  fence_before();
  __syncthreads();
  if (warp == 0) {
    fence_after();
    tmem_dealloc(tmem, tmem_cols);
  }
}

// Sum the slices of every tile that stream-K split between CTAs, in CTA order,
// and apply the epilogue. blockIdx.y + 1 = CTA boundary b; the tile holding it
// is handled by its lowest boundary. Thread = (token, 32-feature chunk).
template <class Epi>
__global__ void __launch_bounds__(128)
gemm_small_reduce_kernel(const float* __restrict__ part, int M_cap, const int* __restrict__ M_dev, int N,
                         SmallPlan p, Epi epi) {
  pdl_wait();  // launched with PDL behind the main kernel: its slices are complete after this
  pdl_trigger();
  const int b = blockIdx.y + 1;
  const int64_t i = sk_begin(b, p);
  if (i % p.nk == 0) return;  // boundary on a tile edge: no tile split here
  const int t = (int)(i / p.nk);
  const int64_t ip = sk_begin(b - 1, p);
  if (ip / p.nk == t && ip % p.nk != 0) return;  // a lower boundary inside this tile handles it
  const int M = M_dev ? min(*M_dev, M_cap) : M_cap;
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  const int m = idx >> 2, q = idx & 3;
  const int f = t * 128 + q * 32;
  if (m >= M || f >= N) return;
  const int c_lo = sk_owner((int64_t)t * p.nk, p), c_hi = sk_owner((int64_t)(t + 1) * p.nk - 1, p);
  float v[32];
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = 0.f;
  // two slices in flight per round; summed strictly in CTA order
  for (int c = c_lo; c <= c_hi; c += 2) {
    const bool two = c + 1 <= c_hi;
    const float4* s0 =
        reinterpret_cast<const float4*>(part + ((int64_t)sk_slot(c, t, p) * M_cap + m) * 128 + q * 32);
    const float4* s1 = two ? reinterpret_cast<const float4*>(part + ((int64_t)sk_slot(c + 1, t, p) * M_cap + m) *
                                                                         128 + q * 32)
                           : s0;
    float4 r0[8], r1[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      r0[j] = __ldcg(s0 + j);
      r1[j] = __ldcg(s1 + j);
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      v[4 * j] += r0[j].x; v[4 * j + 1] += r0[j].y; v[4 * j + 2] += r0[j].z; v[4 * j + 3] += r0[j].w;
    }
    if (two) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        v[4 * j] += r1[j].x; v[4 * j + 1] += r1[j].y; v[4 * j + 2] += r1[j].z; v[4 * j + 3] += r1[j].w;
      }
    }
  }
  epi.template apply<32>(m, f, v);
}

}  // namespace tc

}  // namespace vllt

#include "gemm_bf16_epi.cuh"

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

// Split-K scratch the caller owns: partial tiles and per-tile counters (zeroed
// once; every launch leaves them zero). max_splits <= 1 disables splitting.
struct SplitKScratch {
  float* part = nullptr;
  int64_t part_bytes = 0;
  int* counters = nullptr;
  int n_counters = 0;
  int max_splits = 0;
};

inline int sm_count() {
  static int cached[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return 148;
  if (!cached[dev]) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cached[dev] = n > 0 ? n : 148;
  }
  return cached[dev];
}

// How many K slices a launch of this shape gets: enough CTAs to cover the SMs
// when the tile grid covers fewer than half of them, at least 4 k-blocks per
// slice, within the scratch. Depends only on (M_cap, N, K) and the scratch, so
// eager runs and graph replays of one shape split alike.
inline int choose_splits(int M_cap, int N, int K, const SplitKScratch* sk) {
  if (!sk || sk->max_splits <= 1 || !sk->part || !sk->counters || M_cap <= 0 || N <= 0) return 1;
  const int tiles = ceil_div(N, tc::BN) * ceil_div(M_cap, tc::BM);
  const int sms = sm_count();
  if (tiles * 2 > sms || tiles > sk->n_counters) return 1;
  int s = std::min(std::min(sms / tiles, (K / tc::BK) / 4), sk->max_splits);
  while (s > 1 && (int64_t)s * tiles * tc::BM * tc::BN * 4 > sk->part_bytes) --s;
  return std::max(s, 1);
}

// The forward pass's GEMM scratch: partial slices / tiles for up to 160 SMs
// and 128 tile counters; `base` (may be null for sizing) holds the partials
// followed by the counters.
inline SplitKScratch forward_splitk_scratch(char* base) {
  SplitKScratch sk;
  // the small-M form's slices (2 per CTA, 256 tokens x 128 fp32) bound the size;
  // the split-K form's 160 partial tiles fit in the same bytes
  sk.part_bytes = 2ll * 160 * 256 * 128 * 4;
  sk.n_counters = 128;
  sk.max_splits = 8;
  sk.part = base ? reinterpret_cast<float*>(base) : nullptr;
  sk.counters = base ? reinterpret_cast<int*>(base + sk.part_bytes) : nullptr;
  return sk;
}

// Up to 4 consecutive 64-wide k sub-blocks per ring stage: each weight row is
// then read in 512-byte runs rather than 128-byte ones (measured: up to 25 %
// faster at 64 tokens, equal at 256).
constexpr int kSmallKsubMax = 4;
// Plan of the small-M form for this shape, or false when it does not apply
// (more than 256 token rows, N not a multiple of 32).
inline bool small_plan(int M_cap, int N, int K, tc::SmallPlan* p) {
  if (M_cap <= 0 || M_cap > 256 || N <= 0 || N % 32 || K % tc::BK) return false;
  int n_pad = 32;
  while (n_pad < M_cap) n_pad *= 2;
  p->n_pad = n_pad;
  p->tiles = ceil_div(N, 128);
  // k sub-blocks per ring stage: as many as keep at least 2 stages in the ring
  int ksub = kSmallKsubMax;
  while (ksub > 1 && ((K / tc::BK) % ksub || 2 * ksub * (tc::SK_W_BYTES + n_pad * 128) > tc::SK_RING_BYTES)) ksub /= 2;
  p->ksub = ksub;
  p->nk = K / (tc::BK * ksub);
  p->total = (int64_t)p->tiles * p->nk;
  p->ctas = (int)std::max<int64_t>(1, std::min<int64_t>(sm_count(), p->total / 2));
  const int stage_bytes = ksub * (tc::SK_W_BYTES + n_pad * 128);
  p->stages = std::min(tc::SK_MAX_STAGES, tc::SK_RING_BYTES / stage_bytes);
  return true;
}
inline int64_t small_scratch_bytes(int M_cap, const tc::SmallPlan& p) { return 2ll * p.ctas * M_cap * 128 * 4; }

// Plan of the cluster split-K form: N / 128 feature tiles too few to cover
// the SMs (at least 2 CTAs per tile fit), at most 8 CTAs per cluster, at least
// 2 iterations per CTA. False when it does not apply.
// How many clusters of S CTAs (each `smem` bytes of dynamic shared memory)
// can be resident at once on this device (cached per device and S; the
// epilogue type does not change the kernel's resources that bound it).
inline int max_active_clusters(int S, int smem) {
  static int cache[32][9] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 32 || S < 1 || S > 8) return 0;
  if (!cache[dev][S]) {
    auto fn = tc::gemm_cluster_kernel<EpiStoreF32>;
    cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, 1024 + tc::SK_RING_BYTES);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(S * 64);
    cfg.blockDim = dim3(tc::SK_THREADS);
    cfg.dynamicSmemBytes = smem;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = S;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, fn, &cfg) != cudaSuccess) {
      cudaGetLastError();
      n = -1;  // unknown: the cluster form is not used
    }
    cache[dev][S] = n;
  }
  return cache[dev][S];
}

// Plan of the cluster split-K form: few N / 128 feature tiles, S (2..8) CTAs
// per tile chosen as large as keeps every cluster resident in one wave and
// at least 2 iterations per CTA. False when it does not apply.
inline bool cluster_plan(int M_cap, int N, int K, tc::ClusterPlan* p) {
  if (M_cap <= 0 || M_cap > 256 || N <= 0 || N % 32 || K % tc::BK) return false;
  const int tiles = ceil_div(N, 128);
  int n_pad = 32;
  while (n_pad < M_cap) n_pad *= 2;
  int ksub = kSmallKsubMax;
  while (ksub > 1 && ((K / tc::BK) % ksub || 2 * ksub * (tc::SK_W_BYTES + n_pad * 128) > tc::SK_RING_BYTES)) ksub /= 2;
  const int nk = K / (tc::BK * ksub);
  const int stage_bytes = ksub * (tc::SK_W_BYTES + n_pad * 128);
  const int stages = std::min(tc::SK_MAX_STAGES, tc::SK_RING_BYTES / stage_bytes);
  if (stages * stage_bytes < n_pad * 128 * 4) return false;  // the staging buffer reuses the ring
  const int smem = 1024 + stages * stage_bytes;
  for (int S = std::min(8, sm_count() / tiles); S >= 2; --S) {
    if (nk < 2 * S) continue;
    if (tiles > max_active_clusters(S, smem)) continue;
    *p = tc::ClusterPlan{tiles, S, ksub, nk, n_pad, stages};
    return true;
  }
  return false;
}

template <class Epi>
inline int gemm_cluster_launch(const void* A, int M_cap, const int* M_dev, const void* W, int N, int K,
                               const Epi& epi, int* err, cudaStream_t st, const tc::ClusterPlan& p) {
  CUtensorMap tw, tx;
  int rc = tc::kmajor_map(&tw, W, N, K, 128);
  if (rc != VLLT_OK) return rc;
  rc = tc::kmajor_map(&tx, A, M_cap, K, p.n_pad);
  if (rc != VLLT_OK) return rc;
  const int smem = 1024 + p.stages * p.ksub * (tc::SK_W_BYTES + p.n_pad * 128);
  static PerDeviceOnce smem_opt_in;  // dynamic shared memory above 48 KB, once per device
  smem_opt_in.run([&] {
    cudaFuncSetAttribute(tc::gemm_cluster_kernel<Epi>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         1024 + tc::SK_RING_BYTES);
  });
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.tiles * p.S);
  cfg.blockDim = dim3(tc::SK_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = p.S;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, tc::gemm_cluster_kernel<Epi>, tw, tx, M_cap, M_dev, N, p, epi, err);
  if (e != cudaSuccess) {
    set_error("gemm_bf16 (cluster split-K): launch failed: %s", cudaGetErrorString(e));
    return VLLT_ERR_CUDA;
  }
  return check_launch("gemm_bf16 (cluster split-K)");
}

template <class Epi>
inline int gemm_small_launch(const void* A, int M_cap, const int* M_dev, const void* W, int N, int K,
                             const Epi& epi, int* err, cudaStream_t st, const tc::SmallPlan& p, float* part) {
  CUtensorMap tw, tx;
  int rc = tc::kmajor_map(&tw, W, N, K, 128);
  if (rc != VLLT_OK) return rc;
  rc = tc::kmajor_map(&tx, A, M_cap, K, p.n_pad);
  if (rc != VLLT_OK) return rc;
  const int smem = 1024 + p.stages * p.ksub * (tc::SK_W_BYTES + p.n_pad * 128) + tc::SK_TBUF_BYTES;
  static PerDeviceOnce smem_opt_in;  // dynamic shared memory above 48 KB, once per device
  smem_opt_in.run([&] {
    cudaFuncSetAttribute(tc::gemm_small_kernel<Epi>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         1024 + tc::SK_RING_BYTES + tc::SK_TBUF_BYTES);
  });
  // both kernels start under PDL: the main kernel's set-up and first weight
  // loads overlap the previous kernel, the reduce kernel waits in place
  cudaError_t e = launch_pdl(tc::gemm_small_kernel<Epi>, dim3(p.ctas), dim3(tc::SK_THREADS), (size_t)smem, st, tw,
                             tx, M_cap, M_dev, N, p, epi, part, err);
  if (e != cudaSuccess) {
    set_error("gemm_bf16 (small M): launch failed: %s", cudaGetErrorString(e));
    return VLLT_ERR_CUDA;
  }
  rc = check_launch("gemm_bf16 (small M)");
  if (rc != VLLT_OK || p.ctas < 2) return rc;
  e = launch_pdl(tc::gemm_small_reduce_kernel<Epi>, dim3(ceil_div(M_cap * 4, 128), p.ctas - 1), dim3(128), 0, st,
                 (const float*)part, M_cap, M_dev, N, p, epi);
  if (e != cudaSuccess) {
    set_error("gemm_bf16 (small M reduce): launch failed: %s", cudaGetErrorString(e));
    return VLLT_ERR_CUDA;
  }
  return check_launch("gemm_bf16 (small M reduce)");
}

// D = A . W^T through an epilogue. A [M_cap][K], W [N][K] bf16, K % 64 == 0.
// `splits` > 0 forces that many K slices of the split-K form (1 = the
// persistent form); 0 picks the form: for M_cap <= 256 the cluster split-K
// form when the feature tiles are few, else small-M stream-K when the scratch
// holds its slices; otherwise split-K when choose_splits says so.
template <class Epi>
inline int gemm_bf16_launch(const void* A, int M_cap, const int* M_dev, const void* W, int N, int K, const Epi& epi,
                     int* err, cudaStream_t st, const SplitKScratch* sk = nullptr, int splits = 0) {
  if (M_cap <= 0 || N <= 0) return VLLT_OK;
  VLLT_REQUIRE(K > 0 && K % tc::BK == 0, "gemm_bf16: K must be a positive multiple of 64 (K=%d)", K);
  VLLT_REQUIRE(((uintptr_t)A & 15) == 0 && ((uintptr_t)W & 15) == 0, "gemm_bf16: operands must be 16-byte aligned");
  VLLT_REQUIRE(err, "gemm_bf16: device error word required");
  CUtensorMap ta, tb;
  int rc = tc::kmajor_map(&ta, A, M_cap, K, tc::BM);
  if (rc != VLLT_OK) return rc;
  rc = tc::kmajor_map(&tb, W, N, K, tc::BN);
  if (rc != VLLT_OK) return rc;
  static PerDeviceOnce smem_opt_in;  // dynamic shared memory above 48 KB, once per device
  smem_opt_in.run([&] {
    cudaFuncSetAttribute(tc::gemm_kernel<Epi>, cudaFuncAttributeMaxDynamicSharedMemorySize, tc::SMEM_BYTES);
    cudaFuncSetAttribute(tc::gemm_persistent_kernel<Epi>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         tc::SMEM_BYTES);
  });
  if (splits <= 0) {
    tc::ClusterPlan cp;
    if (cluster_plan(M_cap, N, K, &cp)) return gemm_cluster_launch(A, M_cap, M_dev, W, N, K, epi, err, st, cp);
    tc::SmallPlan sp;
    if (sk && sk->part && small_plan(M_cap, N, K, &sp) && small_scratch_bytes(M_cap, sp) <= sk->part_bytes)
      return gemm_small_launch(A, M_cap, M_dev, W, N, K, epi, err, st, sp, sk->part);
    splits = choose_splits(M_cap, N, K, sk);
  }
  const int64_t tiles = (int64_t)ceil_div(N, tc::BN) * ceil_div(M_cap, tc::BM);
  VLLT_REQUIRE(tiles < (1ll << 31), "gemm_bf16: too many tiles");
  if (splits == 1) {  // persistent: one CTA per SM (at most one per tile)
    const unsigned ctas = (unsigned)std::min<int64_t>(tiles, sm_count());
    VLLT_LAUNCH(ctas, tc::P_THREADS, tc::SMEM_BYTES, st, tc::gemm_persistent_kernel<Epi>)(ta, tb, M_cap, M_dev, N, K,
                                                                                         epi, err);
    return check_launch("gemm_bf16");
  }
  VLLT_REQUIRE(sk && sk->part && sk->counters && tiles <= sk->n_counters &&
                   splits * tiles * tc::BM * tc::BN * 4 <= sk->part_bytes && splits <= K / tc::BK,
               "gemm_bf16: split-K scratch too small for %d slices of %lld tiles (or more slices than k-blocks)",
               splits, (long long)tiles);
  const tc::SplitK ks{sk->part, sk->counters};
  dim3 grid((unsigned)tiles, 1, splits);
  VLLT_LAUNCH(grid, 128, tc::SMEM_BYTES, st, tc::gemm_kernel<Epi>)(ta, tb, M_cap, M_dev, N, K, epi, err, ks);
  return check_launch("gemm_bf16");
}

}  // namespace vllt

