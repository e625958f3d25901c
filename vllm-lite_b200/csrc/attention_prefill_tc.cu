// Paged prefill / verify attention on the tcgen05 tensor cores (bf16,
// head_dim 128, block_size 16, GQA group NREP in {1, 2, 4, 8}).
//
// Same semantics as the generic kernel (paged_attention, vllmlite/attention.py:59-98,
// causal mask of :87-94) for the multi-token query tiles of a ragged batch.
// A CTA owns one KV head and 128 query rows = (128 / NREP positions) x NREP
// heads of the group, position-major, so every K/V tile it loads serves all
// heads of the group. Warp-specialized, 6 warps:
//   warp 4 (loads): Q once by 3-D TMA (one box per 64-wide half of head_dim),
//        then per 128-key tile the K and V blocks (2-D boxes per 16-token block
//        and d half; blocks past the context or with a bad id read the
//        out-of-range zero fill) into separate 2-stage K and V rings;
//   warp 5 (MMA): S_j = Q K_j^T (M128 N128 K16 x 8) into one of two TMEM S
//        buffers, issued one tile ahead so it runs under the softmax of the
//        tile before; O += P_j V_j (V MN-major) into TMEM once P_j is ready;
//   warps 0-3 (softmax, thread = row = TMEM lane): the row's 128 scores in
//        registers, causal mask on the diagonal tile, p = 2^(s*scale - m) on
//        MUFU, P as bf16 into shared memory (swizzled K-major A operand);
//        O is rescaled in TMEM only when the running max grows by > 2^8.
// Q, P, K and V are 128B-swizzled. All waits are bounded; no clusters, no multicast.

#include <cuda.h>

#include "gemm_bf16_tc.cuh"
#include "ops.cuh"

namespace vllt {

namespace {

using namespace tc;

constexpr int kD = 128, kBS = 16, kKeys = 128, kRows = 128;
constexpr int kHalf = kRows * 128;           // one [128 rows][128 B] operand region: 16 KB
constexpr int kTileBytes = 2 * kHalf;        // K or V tile (two d halves): 32 KB
constexpr int kStageBytes = 2 * kTileBytes;  // K + V: 64 KB
constexpr int kSmemBytes = 1024 + 2 * kHalf /*Q*/ + 2 * kHalf /*P*/ + 2 * kStageBytes;  // 197,632

struct PrefillParams {
  const int32_t* tables;
  int W;
  const int32_t* cu_q;
  const int32_t* ctx;
  const int32_t* item_seq;
  const int32_t* item_q0;
  const int32_t* n_items;
  int items_per_seq, num_seqs;
  int H, n_kv, num_blocks;
  int64_t cache_rows;  // num_blocks * n_kv * 16: the row just past the cache (zero fill)
  float qscale;        // softmax scale * log2(e)
  __nv_bfloat16* out;  // [T][H][128]
  int* err;
};

// K-major, 128B-swizzled operand: 8-row groups 1024 B apart.
__device__ __forceinline__ uint64_t desc_kmajor(const void* p) { return smem_desc(p); }
// MN-major, 128B-swizzled operand (V): 64-element N atoms 16 KB apart (LBO),
// 8-row K groups 1024 B apart (SBO).
__device__ __forceinline__ uint64_t desc_mnmajor(const void* p) {
  const uint64_t a = (saddr(p) >> 4) & 0x3FFFu;
  return a | ((uint64_t)(kHalf >> 4) << 16) | (64ull << 32) | (1ull << 46) | (2ull << 61);
}
// kind::f16, fp32 accumulate, bf16 A/B, M128 N128; b_mn selects an MN-major B.
template <bool B_MN>
constexpr uint32_t idesc128() {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((B_MN ? 1u : 0u) << 16) | ((uint32_t)(128 >> 3) << 17) |
         ((uint32_t)(128 >> 4) << 24);
}
#ifdef VLLT_SIMT_HOST
// the host emulation's equivalents (tests/simt_include/simt_tc.h)
template <bool B_MN>
inline void umma(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t acc) {
  ::simt::tensor::mma_f16(tmem_d, a, b, idesc128<B_MN>(), acc);
}
inline void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y, int z) {
  ::simt::tensor::tma_load(dst, map, bar, x, y, z);
}
inline void tmem_st32(uint32_t taddr, const float (&v)[32]) {
  uint32_t r[32];
  for (int i = 0; i < 32; ++i) r[i] = __float_as_uint(v[i]);
  ::simt::tensor::tmem_st32(taddr, r);
}
inline void tmem_ld32_nowait(uint32_t taddr, uint32_t* r) { ::simt::tensor::tmem_ld32(taddr, r); }
inline void tmem_wait_ld() {}
inline void fence_proxy_async() {}
inline float ex2(float x) { return ::simt::tensor::ex2_ftz(x); }
#else
template <bool B_MN>
__device__ __forceinline__ void umma(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n"
      ::"r"(tmem_d), "l"(a), "l"(b), "r"(idesc128<B_MN>()), "r"(acc));
}
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];"
      ::"r"(saddr(dst)), "l"(map), "r"(x), "r"(y), "r"(z), "r"(saddr(bar))
      : "memory");
}
// 32 columns of this thread's TMEM lane into r[0..31]; complete after tmem_wait_ld().
__device__ __forceinline__ void tmem_ld32_nowait(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// generic-proxy writes to shared memory -> visible to the tensor core's reads
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
      ::"r"(taddr), "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
        "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
        "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
        "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
        "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
        "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
        "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
        "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
        "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
        "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
        "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31])));
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// exp2 on the MUFU unit (flush-to-zero: scores below 2^-126 count as 0)
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
#endif

// The running max a row's probabilities are taken against moves only when a
// tile's max exceeds it by more than 2^8 (log2 units): until then P <= 256,
// exact in bf16's exponent range, and O needs no rescale. The result O / l
// does not depend on which max was used.
constexpr float kRescaleLog2 = 8.0f;

template <int NREP>
__global__ void __launch_bounds__(192, 1)
prefill_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                  const __grid_constant__ CUtensorMap tv, PrefillParams p) {
  constexpr int QP = kRows / NREP;  // query positions per CTA
  VLLT_DYNAMIC_SMEM(smem_raw, 1024);
  unsigned char* smem = smem_raw + ((1024 - (saddr(smem_raw) & 1023)) & 1023);
  unsigned char* q_s = smem;                // 2 halves [128 rows][128 B]
  unsigned char* p_s = q_s + 2 * kHalf;     // 2 key halves [128 rows][128 B]
  unsigned char* k_s = p_s + 2 * kHalf;     // 2 stages x K tile (2 d halves)
  unsigned char* v_s = k_s + 2 * kTileBytes;  // 2 stages x V tile
  __shared__ uint64_t bar_q, k_full[2], k_empty[2], v_full[2], v_empty[2], s_full[2], p_full, o_done, drain;
  __shared__ uint32_t tmem_s;
  __shared__ volatile int abort_s;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int kvh = blockIdx.x;
  int s, q0;
  if (p.item_seq) {  // work list: heaviest (latest) items first
    const int n = *p.n_items;
    if ((int)blockIdx.y >= n) return;
    const int it = n - 1 - (int)blockIdx.y;
    s = p.item_seq[it];
    q0 = p.item_q0[it];
  } else {
    s = blockIdx.y / p.items_per_seq;
    q0 = (p.items_per_seq - 1 - (int)(blockIdx.y % p.items_per_seq)) * QP;
    if (s >= p.num_seqs) return;
  }
  const int tok0 = p.cu_q[s];
  const int qlen = p.cu_q[s + 1] - tok0;
  if (q0 >= qlen) return;
  const int ctx = min(p.ctx[s], p.W * kBS);
  const int first_qpos = ctx - qlen + q0;
  const int last_qpos = min(first_qpos + QP - 1, ctx - 1);
  const int n_tiles = last_qpos / kKeys + 1;
  const int32_t* table = p.tables + (int64_t)s * p.W;

  if (tid == 0) {
    mbar_init(&bar_q, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&s_full[i], 1);
    }
    mbar_init(&p_full, 128);
    mbar_init(&o_done, 1);
    mbar_init(&drain, 1);
    flag_write(&abort_s, 0);
    mbar_fence_init();
  }
  if (warp == 0) {
    tmem_alloc(&tmem_s, 512);
    tmem_relinquish();
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = tmem_s, t_O = tmem + 256;  // S buffers at columns 0 and 128

  if (warp == 4) {
    if (lane == 0) {  // ---- loads: Q once, then K_j and V_j into 2-stage rings ----
      mbar_expect_tx(&bar_q, 2 * kHalf);
      tma_load_3d(q_s, &tq, &bar_q, 0, kvh * NREP, tok0 + q0);
      tma_load_3d(q_s + kHalf, &tq, &bar_q, 64, kvh * NREP, tok0 + q0);
      int jk = 0, jv = 0;  // tiles issued per ring
      bool failed = false;
      for (int j = 0; j < n_tiles && !failed; ++j) {
        int y[kKeys / kBS];
#pragma unroll
        for (int b = 0; b < kKeys / kBS; ++b) {
          const int kb = j * (kKeys / kBS) + b;  // block index within the sequence
          const int blk = (kb * kBS < ctx) ? table[kb] : -1;
          y[b] = (blk >= 0 && blk < p.num_blocks) ? (blk * p.n_kv + kvh) * kBS : (int)p.cache_rows;
        }
        const int st = j & 1;
        if (j >= 2 && !mbar_wait_or_abort(&k_empty[st], ((j >> 1) & 1) ^ 1, &abort_s)) {
          failed = true;
          break;
        }
        mbar_expect_tx(&k_full[st], kTileBytes);
#pragma unroll
        for (int b = 0; b < kKeys / kBS; ++b) {
          unsigned char* dst = k_s + st * kTileBytes + b * (kBS * 128);
          tma_load_2d(dst, &tk, &k_full[st], 0, y[b]);
          tma_load_2d(dst + kHalf, &tk, &k_full[st], 64, y[b]);
        }
        jk = j + 1;
        if (j >= 2 && !mbar_wait_or_abort(&v_empty[st], ((j >> 1) & 1) ^ 1, &abort_s)) {
          failed = true;
          break;
        }
        mbar_expect_tx(&v_full[st], kTileBytes);
#pragma unroll
        for (int b = 0; b < kKeys / kBS; ++b) {
          unsigned char* dst = v_s + st * kTileBytes + b * (kBS * 128);
          tma_load_2d(dst, &tv, &v_full[st], 0, y[b]);
          tma_load_2d(dst + kHalf, &tv, &v_full[st], 64, y[b]);
        }
        jv = j + 1;
      }
      if (failed) {  // let the copies in flight land before the CTA can exit (bounded)
        atomicOr(p.err, 4);
        flag_write(&abort_s, 1);
        (void)mbar_wait(&bar_q, 0);
        for (int t = max(0, jk - 2); t < jk; ++t) (void)mbar_wait(&k_full[t & 1], (t >> 1) & 1);
        for (int t = max(0, jv - 2); t < jv; ++t) (void)mbar_wait(&v_full[t & 1], (t >> 1) & 1);
      }
    }
  } else if (warp == 5) {
    if (lane == 0) {  // ---- MMA: S_{j+1} = Q K^T ahead of the softmax, then O += P_j V_j ----
      bool ok = mbar_wait_or_abort(&bar_q, 0, &abort_s) && mbar_wait_or_abort(&k_full[0], 0, &abort_s);
      int issued = 0;
      auto issue_s = [&](int j) {
        fence_after();
        const unsigned char* kt = k_s + (j & 1) * kTileBytes;
        const uint32_t t_S = tmem + (j & 1) * 128;
#pragma unroll
        for (int k = 0; k < kD / 16; ++k) {
          const int h = k >> 2, off = (k & 3) * 32;
          umma<false>(t_S, desc_kmajor(q_s + h * kHalf + off), desc_kmajor(kt + h * kHalf + off), k > 0 ? 1u : 0u);
        }
        mma_commit(&s_full[j & 1]);
        mma_commit(&k_empty[j & 1]);
        ++issued;
      };
      if (ok) issue_s(0);
      for (int j = 0; j < n_tiles && ok; ++j) {
        // S buffer (j+1)&1 was last read by the softmax of tile j-1, complete since p_full(j-1)
        if (j + 1 < n_tiles) {
          if (!mbar_wait_or_abort(&k_full[(j + 1) & 1], ((j + 1) >> 1) & 1, &abort_s)) {
            ok = false;
            break;
          }
          issue_s(j + 1);
        }
        if (!mbar_wait_or_abort(&p_full, j & 1, &abort_s) ||
            !mbar_wait_or_abort(&v_full[j & 1], (j >> 1) & 1, &abort_s)) {
          ok = false;
          break;
        }
        fence_after();
        const unsigned char* vt = v_s + (j & 1) * kTileBytes;
#pragma unroll
        for (int k = 0; k < kKeys / 16; ++k) {
          const int h = k >> 2, off = (k & 3) * 32;
          umma<true>(t_O, desc_kmajor(p_s + h * kHalf + off), desc_mnmajor(vt + k * 16 * 128),
                     (j > 0 || k > 0) ? 1u : 0u);
        }
        mma_commit(&v_empty[j & 1]);
        mma_commit(&o_done);
        ++issued;
      }
      if (!ok) {
        atomicOr(p.err, 4);
        flag_write(&abort_s, 1);
      }
      if (issued > 0) {  // every MMA finished before the columns are freed
        mma_commit(&drain);
        (void)mbar_wait(&drain, 0);
      }
    }
  } else {  // ---- softmax warps 0-3: thread = query row = TMEM lane ----
    const int row = tid;
    const int qpos = first_qpos + row / NREP;
    const uint32_t lane_base = (uint32_t)(warp * 32) << 16;
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    for (int j = 0; j < n_tiles; ++j) {
      if (!__all_sync(0xffffffffu, mbar_wait_or_abort(&s_full[j & 1], (j >> 1) & 1, &abort_s))) {
        ok = false;
        break;
      }
      fence_after();
      float v[kKeys];
      {
        const uint32_t ta = tmem + (j & 1) * 128 + lane_base;
        uint32_t r[kKeys];
#pragma unroll
        for (int c = 0; c < kKeys; c += 32) tmem_ld32_nowait(ta + c, r + c);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < kKeys; ++i) v[i] = __uint_as_float(r[i]);
      }
      const int key0 = j * kKeys;
      if (key0 + kKeys - 1 > first_qpos) {  // diagonal tile: mask keys past this row's position
#pragma unroll
        for (int i = 0; i < kKeys; ++i)
          if (key0 + i > qpos) v[i] = -INFINITY;
      }
      float mx = -INFINITY;
#pragma unroll
      for (int i = 0; i < kKeys; ++i) mx = fmaxf(mx, v[i]);
      mx *= p.qscale;  // scale > 0: max(s) * scale = max(s * scale)
      float m_use = m_run, alpha = 1.f;
      if (mx > m_run + kRescaleLog2) {  // also the first tile with a finite max (m_run = -inf)
        m_use = mx;
        alpha = m_run == -INFINITY ? 0.f : ex2(m_run - mx);
      }
      float sum = 0.f;
      uint32_t pk[kKeys / 2];
#pragma unroll
      for (int i = 0; i < kKeys; i += 2) {
        const float p0 = ex2(fmaf(v[i], p.qscale, -m_use)), p1 = ex2(fmaf(v[i + 1], p.qscale, -m_use));
        sum += p0 + p1;
        const __nv_bfloat162 b = __floats2bfloat162_rn(p0, p1);
        pk[i / 2] = *reinterpret_cast<const uint32_t*>(&b);
      }
      // P_{j-1} V_{j-1} complete: O is stable and the P buffer free
      if (j > 0 && !__all_sync(0xffffffffu, mbar_wait_or_abort(&o_done, (j - 1) & 1, &abort_s))) {
        ok = false;
        break;
      }
      fence_after();
      if (j > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll 1
        for (int c = 0; c < kD; c += 32) {
          float o[32];
          tmem_ld32(t_O + lane_base + c, o);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] *= alpha;
          tmem_st32(t_O + lane_base + c, o);
        }
      }
      l_run = l_run * alpha + sum;
      m_run = m_use;
#pragma unroll
      for (int c = 0; c < kKeys; c += 8) {  // 8 keys = one 16-byte chunk of the swizzled row
        const int chunk = (c & 63) >> 3;
        unsigned char* prow = p_s + (c >> 6) * kHalf + row * 128;
        *reinterpret_cast<uint4*>(prow + ((chunk ^ (row & 7)) << 4)) =
            make_uint4(pk[c / 2], pk[c / 2 + 1], pk[c / 2 + 2], pk[c / 2 + 3]);
      }
      fence_proxy_async();  // P: generic writes -> MMA reads
      fence_before();
      mbar_arrive(&p_full);
    }
    if (!ok) {
      if (lane == 0) atomicOr(p.err, 4);
      flag_write(&abort_s, 1);
    } else if (__all_sync(0xffffffffu, mbar_wait_or_abort(&o_done, (n_tiles - 1) & 1, &abort_s))) {
      fence_after();  // epilogue: O / l -> bf16 rows
      const int pos = q0 + row / NREP;
      const int head = kvh * NREP + row % NREP;
      const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
      __nv_bfloat16* dst = p.out + ((int64_t)(tok0 + pos) * p.H + head) * kD;
#pragma unroll 1
      for (int c = 0; c < kD; c += 32) {
        float o[32];
        tmem_ld32(t_O + lane_base + c, o);
        if (pos < qlen) {
#pragma unroll
          for (int i = 0; i < 32; i += 8) {
            __nv_bfloat162 a = __floats2bfloat162_rn(o[i] * inv, o[i + 1] * inv);
            __nv_bfloat162 b = __floats2bfloat162_rn(o[i + 2] * inv, o[i + 3] * inv);
            __nv_bfloat162 cc = __floats2bfloat162_rn(o[i + 4] * inv, o[i + 5] * inv);
            __nv_bfloat162 d = __floats2bfloat162_rn(o[i + 6] * inv, o[i + 7] * inv);
            uint4 w;
            w.x = *reinterpret_cast<uint32_t*>(&a); w.y = *reinterpret_cast<uint32_t*>(&b);
            w.z = *reinterpret_cast<uint32_t*>(&cc); w.w = *reinterpret_cast<uint32_t*>(&d);
            *reinterpret_cast<uint4*>(dst + c + i) = w;
          }
        }
      }
    } else {
      if (lane == 0) atomicOr(p.err, 4);
      flag_write(&abort_s, 1);
    }
  }
  fence_before();
  __syncthreads();
  if (warp == 0) {
    fence_after();
    tmem_dealloc(tmem, 512);
  }
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

int encode(CUtensorMap* m, int rank, const void* base, const cuuint64_t* dims, const cuuint64_t* strides,
           const cuuint32_t* box) {
  auto enc = reinterpret_cast<EncodeTiledFn>(tc::encode_fn());
  if (!enc) {
    set_error("prefill attention: cuTensorMapEncodeTiled unavailable");
    return VLLT_ERR_CUDA;
  }
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, const_cast<void*>(base), dims, strides, box,
                         estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("prefill attention: cuTensorMapEncodeTiled failed (%d)", (int)r);
    return VLLT_ERR_CUDA;
  }
  return VLLT_OK;
}

template <int NREP>
int launch_prefill(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv, const PrefillParams& p,
                   int items, cudaStream_t st) {
  static PerDeviceOnce smem_opt_in;  // dynamic shared memory above 48 KB, once per device
  smem_opt_in.run([&] {
    cudaFuncSetAttribute(prefill_tc_kernel<NREP>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
  });
  VLLT_LAUNCH(dim3(p.n_kv, items), 192, kSmemBytes, st, prefill_tc_kernel<NREP>)(tq, tk, tv, p);
  return check_launch("prefill attention (tcgen05)");
}

}  // namespace

bool prefill_tc_supported(const AttnCall& c) {
  const int n_rep = c.H / c.n_kv;
  return c.dtype == VLLT_BF16 && c.D == kD && c.bs == kBS && (n_rep == 1 || n_rep == 2 || n_rep == 4 || n_rep == 8);
}

int prefill_tc_positions(int n_rep) { return kRows / n_rep; }

// Multi-token tiles of 128 / n_rep query positions. q and out are [T_rows][H][128].
int prefill_tc_pass(const AttnCall& c, int T_rows, const int32_t* item_seq, const int32_t* item_q0,
                    const int32_t* n_items, int items_cap, int items_per_seq, int num_seqs, int* err,
                    cudaStream_t st) {
  if (items_cap <= 0) return VLLT_OK;
  VLLT_REQUIRE(err, "prefill attention: error word required");
  const int n_rep = c.H / c.n_kv;
  CUtensorMap tq, tk, tv;
  {
    const cuuint64_t dims[3] = {(cuuint64_t)kD, (cuuint64_t)c.H, (cuuint64_t)std::max(T_rows, 1)};
    const cuuint64_t strides[2] = {(cuuint64_t)kD * 2, (cuuint64_t)c.H * kD * 2};
    const cuuint32_t box[3] = {64, (cuuint32_t)n_rep, (cuuint32_t)(kRows / n_rep)};
    int rc = encode(&tq, 3, c.q, dims, strides, box);
    if (rc != VLLT_OK) return rc;
  }
  const int64_t rows = (int64_t)c.num_blocks * c.n_kv * kBS;
  {
    const cuuint64_t dims[2] = {(cuuint64_t)kD, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)kD * 2};
    const cuuint32_t box[2] = {64, (cuuint32_t)kBS};
    int rc = encode(&tk, 2, c.kc, dims, strides, box);
    if (rc != VLLT_OK) return rc;
    rc = encode(&tv, 2, c.vc, dims, strides, box);
    if (rc != VLLT_OK) return rc;
  }
  PrefillParams p{};
  p.tables = c.tables; p.W = c.W; p.cu_q = c.cu_q; p.ctx = c.ctx;
  p.item_seq = item_seq; p.item_q0 = item_q0; p.n_items = n_items;
  p.items_per_seq = items_per_seq; p.num_seqs = num_seqs;
  p.H = c.H; p.n_kv = c.n_kv; p.num_blocks = c.num_blocks; p.cache_rows = rows;
  p.qscale = c.scale * 1.4426950408889634f;
  p.out = reinterpret_cast<__nv_bfloat16*>(c.out);
  p.err = err;
  switch (n_rep) {
    case 1: return launch_prefill<1>(tq, tk, tv, p, items_cap, st);
    case 2: return launch_prefill<2>(tq, tk, tv, p, items_cap, st);
    case 4: return launch_prefill<4>(tq, tk, tv, p, items_cap, st);
    default: return launch_prefill<8>(tq, tk, tv, p, items_cap, st);
  }
}

}  // namespace vllt
