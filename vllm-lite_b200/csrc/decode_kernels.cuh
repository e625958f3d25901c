// Device code of the bf16 / head_dim 128 / block 16 decode attention kernel
// (launched by attention_decode.cu): its parameters, the mbarrier and
// tensor-map helpers and the kernel. Under the host emulation
// (VLLT_SIMT_HOST, tests/simt_host.h) the helpers written in inline PTX have
// host equivalents, so the CPU tests can run the kernel's own code.
#pragma once

#include <math.h>
#include <stdint.h>

#include <cuda.h>

#include "device_common.cuh"
#ifdef VLLT_SIMT_HOST
#include <simt_tc.h>
#endif

namespace vllt {
namespace dk {

constexpr int kD = 128;
constexpr int kBS = 16;
constexpr int kWarps = 4;
constexpr int kStages = 2;
constexpr int kBox = 16 * 128;            // one 16 x 64 bf16 box: 2 KB
constexpr int kStageBytes = 4 * kBox;     // K lo, K hi, V lo, V hi
constexpr uint64_t kWaitNs = 1000000000;  // bounded mbarrier wait: 1 s

struct DecodeParams {
  const __nv_bfloat16* q;  // [T][H][128]
  __nv_bfloat16* out;      // [T][H][128]
  const int32_t* tables;
  int W;
  const int32_t* cu_q;
  const int32_t* ctx;
  const int32_t* item_seq;  // decode list, or NULL: item = sequence
  const int32_t* n_items;
  int num_seqs;
  int H, n_kv, num_blocks;
  float qscale;       // softmax scale * log2(e)
  int split_blocks;   // blocks per split; 0 = whole context in one CTA
  float* ws_o;        // [splits][P_cap][H][128]  (P_cap = sequence capacity)
  float* ws_ml;       // [splits][P_cap][H][2] (max in natural-log units, sum)
  int P_cap;
  int* err;           // bit 2: a bounded wait expired
  uint64_t wait_ns;   // limit of every mbarrier wait
  int stall_block;    // test: table index whose stage is armed with no copy (-1: none)
};

#ifdef VLLT_SIMT_HOST
// The host emulation's equivalents of the mbarrier and TMA operations below
// (tests/simt_include/simt_tc.h, shared with the tensor-core kernels): an
// mbarrier word holds the pending transaction bytes, the pending arrivals,
// the arrival count and the phase bit; a tensor-map load copies its box at
// once (with the map's swizzle) and completes its bytes; the clock that
// bounds the waits is virtual.
inline uint32_t saddr(const void* p) { return ::simt::tensor::saddr(p); }
inline void mbar_init(uint64_t* bar, unsigned count) { ::simt::tensor::mbar_init(bar, count); }
inline void mbar_fence_init() {}
inline void mbar_expect_tx(uint64_t* bar, unsigned bytes) { ::simt::tensor::mbar_expect_tx(bar, bytes); }
inline void mbar_arrive(uint64_t* bar) { ::simt::tensor::mbar_arrive(bar); }
inline bool mbar_try_wait(uint64_t* bar, unsigned parity) { return ::simt::tensor::mbar_try_wait(bar, parity); }
inline uint64_t global_ns() { return ::simt::tensor::global_ns(); }
inline void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  ::simt::tensor::tma_load(dst, map, bar, x, y, 0);
}
#else
__device__ __forceinline__ uint32_t saddr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(saddr(bar)), "r"(count) : "memory");
}
// Makes the barrier initialisations visible before any other thread uses them.
__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(saddr(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(saddr(bar)) : "memory");
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
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(saddr(dst)), "l"(map), "r"(x), "r"(y), "r"(saddr(bar))
      : "memory");
}
#endif
// Wait for `parity` with a time limit; false if it expired.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, unsigned parity, uint64_t limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  while (!mbar_try_wait(bar, parity))
    if (global_ns() - t0 > limit_ns) return false;
  return true;
}
__device__ __forceinline__ float2 bf2(uint32_t w) {
  return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
}

// Byte offset of 16-byte chunk c of row r in a 128B-swizzled 1024-aligned box.
__device__ __forceinline__ int swz(int r, int c) { return r * 128 + ((c ^ (r & 7)) << 4); }

template <int NREP>
__global__ void __launch_bounds__(kWarps * 32, 3)
decode_kernel(const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tv, DecodeParams p) {
  VLLT_DYNAMIC_SMEM(smem_raw, 1024);
  // 1024-align the stage ring (the swizzle pattern is defined on 1 KB atoms)
  unsigned char* smem = smem_raw + ((1024 - (saddr(smem_raw) & 1023)) & 1023);
  unsigned char* ring = smem;                                            // [warps][stages][8 KB]
  float* q_s = reinterpret_cast<float*>(ring + kWarps * kStages * kStageBytes);  // [NREP][128]
  float2* p_s = reinterpret_cast<float2*>(q_s + NREP * kD);             // [warps][16][NREP] (p, p)
  uint64_t* bars = reinterpret_cast<uint64_t*>(p_s + kWarps * kBS * NREP);  // [warps][stages]

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int kvh = blockIdx.x;
  int s;
  if (p.item_seq) {
    if ((int)blockIdx.y >= *p.n_items) return;
    s = p.item_seq[blockIdx.y];
  } else {
    s = blockIdx.y;
    if (s >= p.num_seqs) return;
  }
  const int t_tok = p.cu_q[s];
  const int ctx = min(p.ctx[s], p.W * kBS);
  const int nblk = (ctx + kBS - 1) / kBS;
  const int split = blockIdx.z;
  int b_begin = 0, b_end = nblk;
  if (p.split_blocks > 0) {
    b_begin = split * p.split_blocks;
    b_end = min(nblk, b_begin + p.split_blocks);
  }
  if (b_begin >= b_end) return;  // uniform; the merge reads only splits < ceil(nblk / split_blocks)

  // barriers first (lane 0 of each warp owns its ring), then q
  if (lane == 0)
    for (int i = 0; i < kStages; ++i) mbar_init(&bars[warp * kStages + i], 1);
  mbar_fence_init();
  for (int i = threadIdx.x; i < NREP * kD; i += blockDim.x) {
    const int h = kvh * NREP + i / kD;
    q_s[i] = __bfloat162float(p.q[((int64_t)t_tok * p.H + h) * kD + i % kD]) * p.qscale;
  }
  __syncthreads();

  const int32_t* table = p.tables + (int64_t)s * p.W;
  unsigned char* my_ring = ring + warp * kStages * kStageBytes;
  uint64_t* my_bars = bars + warp * kStages;
  // this warp's blocks: b_begin + warp + j * kWarps
  const int my_n = (b_end - b_begin - warp + kWarps - 1) / kWarps;

  auto issue = [&](int j) {  // lane 0 only
    const int b = b_begin + warp + j * kWarps;
    const int st = j % kStages;
    uint64_t* bar = &my_bars[st];
    const int blk = table[b];
    if (blk < 0 || blk >= p.num_blocks) {
      mbar_arrive(bar);  // completes the phase with nothing loaded; consumers mask the block
      return;
    }
    const int y = (blk * p.n_kv + kvh) * kBS;
    unsigned char* dst = my_ring + st * kStageBytes;
    mbar_expect_tx(bar, kStageBytes);
    if (b == p.stall_block) return;  // test: bytes promised, no copy issued, the wait expires
    tma_load_2d(dst, &tk, bar, 0, y);
    tma_load_2d(dst + kBox, &tk, bar, 64, y);
    tma_load_2d(dst + 2 * kBox, &tv, bar, 0, y);
    tma_load_2d(dst + 3 * kBox, &tv, bar, 64, y);
  };
  if (lane == 0)
    for (int j = 0; j < min(kStages, my_n); ++j) issue(j);
  __syncwarp();

  float m_run[NREP], l_run[NREP];
  float2 acc[NREP][2];  // this lane's 4 output columns per head, as two pairs
#pragma unroll
  for (int h = 0; h < NREP; ++h) {
    m_run[h] = -INFINITY;
    l_run[h] = 0.f;
    acc[h][0] = acc[h][1] = make_float2(0.f, 0.f);
  }

  const int tq = lane & 15, half = lane >> 4;
  int koff[8];  // this lane's 8 score-loop chunk offsets (row tq of a swizzled box)
#pragma unroll
  for (int c = 0; c < 8; ++c) koff[c] = half * kBox + swz(tq, c);
  const int c16 = lane >> 1;  // P.V: 16-byte chunk of the 256-byte row this lane reads
  const int vbase = 2 * kBox + (c16 >> 3) * kBox + (lane & 1) * 8;
  bool failed = false;
  int j = 0;
  for (; j < my_n; ++j) {
    const int st = j % kStages;
    const int b = b_begin + warp + j * kWarps;
    if (!mbar_wait(&my_bars[st], (j / kStages) & 1, p.wait_ns)) {
      failed = true;
      break;
    }
    const unsigned char* stage = my_ring + st * kStageBytes;
    const int blk = table[b];
    const bool blk_ok = blk >= 0 && blk < p.num_blocks;

    // ---- scores: token tq, columns [half*64, half*64+64) -------------------------
    float2 sc2[NREP];
#pragma unroll
    for (int h = 0; h < NREP; ++h) sc2[h] = make_float2(0.f, 0.f);
    const float* qh = q_s + half * 64;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const uint4 kw = *reinterpret_cast<const uint4*>(stage + koff[c]);
      const float2 k0 = bf2(kw.x), k1 = bf2(kw.y), k2 = bf2(kw.z), k3 = bf2(kw.w);
#pragma unroll
      for (int h = 0; h < NREP; ++h) {
        const float4 qa = *reinterpret_cast<const float4*>(qh + h * kD + c * 8);
        const float4 qb = *reinterpret_cast<const float4*>(qh + h * kD + c * 8 + 4);
        sc2[h] = __ffma2_rn(k0, make_float2(qa.x, qa.y), sc2[h]);
        sc2[h] = __ffma2_rn(k1, make_float2(qa.z, qa.w), sc2[h]);
        sc2[h] = __ffma2_rn(k2, make_float2(qb.x, qb.y), sc2[h]);
        sc2[h] = __ffma2_rn(k3, make_float2(qb.z, qb.w), sc2[h]);
      }
    }
    const bool valid = blk_ok && (b * kBS + tq < ctx);
    float pr[NREP];
#pragma unroll
    for (int h = 0; h < NREP; ++h) {
      float x = sc2[h].x + sc2[h].y;
      x += __shfl_xor_sync(0xffffffffu, x, 16);
      x = valid ? x : -INFINITY;
      float mb = x;
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) mb = fmaxf(mb, __shfl_xor_sync(0xffffffffu, mb, o));
      const float mn = fmaxf(m_run[h], mb);
      const float alpha = m_run[h] == -INFINITY ? 0.f : exp2f(m_run[h] - mn);
      pr[h] = valid ? exp2f(x - mn) : 0.f;
      float sum = pr[h];
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
      l_run[h] = fmaf(l_run[h], alpha, sum);
      m_run[h] = mn;
      const float2 a2 = make_float2(alpha, alpha);
      acc[h][0] = __fmul2_rn(acc[h][0], a2);
      acc[h][1] = __fmul2_rn(acc[h][1], a2);
    }
    float2* pw = p_s + warp * kBS * NREP;
    if (half == 0) {
#pragma unroll
      for (int h = 0; h < NREP; ++h) pw[tq * NREP + h] = make_float2(pr[h], pr[h]);
    }
    __syncwarp();

    // ---- P.V: lane owns columns 4*lane .. 4*lane+3 ---------------------------------
    const unsigned char* vrow = stage + vbase;
#pragma unroll
    for (int t = 0; t < kBS; ++t) {
      const uint2 vw = *reinterpret_cast<const uint2*>(vrow + t * 128 + (((c16 & 7) ^ (t & 7)) << 4));
      const float2 v01 = bf2(vw.x), v23 = bf2(vw.y);
      if constexpr (NREP == 1) {
        const float2 pp = pw[t];
        acc[0][0] = __ffma2_rn(pp, v01, acc[0][0]);
        acc[0][1] = __ffma2_rn(pp, v23, acc[0][1]);
      } else {
#pragma unroll
        for (int h = 0; h < NREP; h += 2) {  // two heads' (p, p) pairs per 16-byte load
          const float4 pq = *reinterpret_cast<const float4*>(&pw[t * NREP + h]);
          const float2 p0 = make_float2(pq.x, pq.y), p1 = make_float2(pq.z, pq.w);
          acc[h][0] = __ffma2_rn(p0, v01, acc[h][0]);
          acc[h][1] = __ffma2_rn(p0, v23, acc[h][1]);
          acc[h + 1][0] = __ffma2_rn(p1, v01, acc[h + 1][0]);
          acc[h + 1][1] = __ffma2_rn(p1, v23, acc[h + 1][1]);
        }
      }
    }
    __syncwarp();  // every lane is done with this stage before it is refilled
    if (lane == 0 && j + kStages < my_n) issue(j + kStages);
  }
  if (failed) {
    if (lane == 0) atomicOr(p.err, 4);
    // let the copies this warp still has in flight land before the CTA exits
    for (int k = j; k < min(my_n, j + kStages); ++k)
      (void)mbar_wait(&my_bars[k % kStages], (k / kStages) & 1, p.wait_ns);
  }

  // ---- merge the four warps (reuse the ring) ---------------------------------------
  __syncthreads();
  float* m_s = reinterpret_cast<float*>(ring);           // [warps][NREP]
  float* l_s = m_s + kWarps * NREP;                       // [warps][NREP]
  float* a_s = l_s + kWarps * NREP;                       // [warps][NREP][128]
  if (lane == 0) {
#pragma unroll
    for (int h = 0; h < NREP; ++h) {
      m_s[warp * NREP + h] = failed ? -INFINITY : m_run[h];
      l_s[warp * NREP + h] = failed ? 0.f : l_run[h];
    }
  }
#pragma unroll
  for (int h = 0; h < NREP; ++h) {
    float* dst = a_s + (warp * NREP + h) * kD + 4 * lane;
    *reinterpret_cast<float4*>(dst) = make_float4(acc[h][0].x, acc[h][0].y, acc[h][1].x, acc[h][1].y);
  }
  __syncthreads();
  constexpr float kLn2 = 0.69314718055994530942f;
  for (int i = threadIdx.x; i < NREP * kD; i += blockDim.x) {
    const int h = i / kD, d = i % kD;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) M = fmaxf(M, m_s[w * NREP + h]);
    float L = 0.f, O = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < kWarps; ++w) {
        const float mw = m_s[w * NREP + h];
        const float e = mw == -INFINITY ? 0.f : exp2f(mw - M);
        L = fmaf(l_s[w * NREP + h], e, L);
        O = fmaf(a_s[(w * NREP + h) * kD + d], e, O);
      }
    }
    const int head = kvh * NREP + h;
    if (p.split_blocks > 0) {
      const int64_t base = ((int64_t)split * p.P_cap + s) * p.H + head;
      p.ws_o[base * kD + d] = L > 0.f ? O / L : 0.f;
      if (d == 0) {
        p.ws_ml[base * 2] = M == -INFINITY ? -INFINITY : M * kLn2;
        p.ws_ml[base * 2 + 1] = L;
      }
    } else {
      p.out[((int64_t)t_tok * p.H + head) * kD + d] = __float2bfloat16_rn(L > 0.f ? O / L : 0.f);
    }
  }
}

template <int NREP>
size_t decode_smem() {
  return 1024 + (size_t)kWarps * kStages * kStageBytes + NREP * kD * 4 + kWarps * kBS * NREP * 8 +
         kWarps * kStages * 8;
}

}  // namespace dk
}  // namespace vllt
