// Paged prefill / verify attention on the tcgen05 tensor cores (bf16,
// head_dim 128, block_size 16, GQA group NREP in {1, 2, 4, 8}).
//
// Same semantics as the generic kernel (paged_attention, vllmlite/attention.py:59-98,
// causal mask of :87-94) for the multi-token query tiles of a ragged batch.
// A CTA owns one KV head and 128 query rows = (128 / NREP positions) x NREP
// heads of the group, position-major, so every K/V tile it loads serves all
// heads of the group.
//
//   Q  : one 3-D TMA load per 64-wide half of head_dim (tokens x heads x d box),
//        128B swizzle -> K-major A operand.
//   K,V: per 16-token block two 2-D TMA boxes (d halves) each; blocks past the
//        context or with a bad id read the out-of-range zero fill. K is the
//        K-major B operand of S = Q K^T; V is the MN-major B operand of O = P V.
//   S  : tcgen05.mma M128 N128 K16 x 8 into tensor memory columns [0, 128).
//   softmax: thread t owns row t (TMEM lane t): two passes over S (max, then
//        p = 2^(s - m)), online across key tiles; P is written as bf16 into
//        shared memory in the swizzled K-major layout.
//   O  : tcgen05.mma (P from shared memory, V) into columns [128, 256); a
//        row's O is rescaled in tensor memory only when its max moved.
// K/V tiles are double buffered (next tile loads while this one is processed).
// All waits are bounded; no clusters, no multicast.

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

template <int NREP>
__global__ void __launch_bounds__(128, 1)
prefill_tc_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                  const __grid_constant__ CUtensorMap tv, PrefillParams p) {
  constexpr int QP = kRows / NREP;  // query positions per CTA
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = smem_raw + ((1024 - (saddr(smem_raw) & 1023)) & 1023);
  unsigned char* q_s = smem;                   // 2 halves [128 rows][128 B]
  unsigned char* p_s = q_s + 2 * kHalf;        // 2 key halves [128 rows][128 B]
  unsigned char* kv_s = p_s + 2 * kHalf;       // 2 stages x (K 2 halves, V 2 halves)
  __shared__ uint64_t bar_q, bar_kv[2], bar_s, bar_o;
  __shared__ uint32_t tmem_s;
  __shared__ int fail_s;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int kvh = blockIdx.x;
  int s, q0;
  if (p.item_seq) {
    if ((int)blockIdx.y >= *p.n_items) return;
    s = p.item_seq[blockIdx.y];
    q0 = p.item_q0[blockIdx.y];
  } else {
    s = blockIdx.y / p.items_per_seq;
    q0 = (blockIdx.y % p.items_per_seq) * QP;
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
    mbar_init(&bar_kv[0], 1);
    mbar_init(&bar_kv[1], 1);
    mbar_init(&bar_s, 1);
    mbar_init(&bar_o, 1);
    fail_s = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(saddr(&tmem_s)), "r"(256));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = tmem_s, t_S = tmem, t_O = tmem + 128;
  const uint32_t lane_base = (uint32_t)(warp * 32) << 16;

  // K/V tile j -> stage j & 1: 8 blocks x (K lo, K hi, V lo, V hi)
  auto load_kv = [&](int j) {
    unsigned char* st = kv_s + (j & 1) * kStageBytes;
    uint64_t* bar = &bar_kv[j & 1];
    mbar_expect_tx(bar, kStageBytes);
#pragma unroll 1
    for (int b = 0; b < kKeys / kBS; ++b) {
      const int kb = j * (kKeys / kBS) + b;  // block index within the sequence
      int blk = (kb * kBS < ctx) ? table[kb] : -1;
      const int y = (blk >= 0 && blk < p.num_blocks) ? (blk * p.n_kv + kvh) * kBS : (int)p.cache_rows;
      unsigned char* kdst = st + b * (kBS * 128);
      tma_load_2d(kdst, &tk, bar, 0, y);
      tma_load_2d(kdst + kHalf, &tk, bar, 64, y);
      tma_load_2d(kdst + kTileBytes, &tv, bar, 0, y);
      tma_load_2d(kdst + kTileBytes + kHalf, &tv, bar, 64, y);
    }
  };

  int issued = 0, consumed = 0;  // K/V tiles (thread 0's bookkeeping for the failure path)
  if (tid == 0) {
    mbar_expect_tx(&bar_q, 2 * kHalf);
    tma_load_3d(q_s, &tq, &bar_q, 0, kvh * NREP, tok0 + q0);
    tma_load_3d(q_s + kHalf, &tq, &bar_q, 64, kvh * NREP, tok0 + q0);
    load_kv(0);
    issued = 1;
    if (n_tiles > 1) {
      load_kv(1);
      issued = 2;
    }
  }

  // this thread's row
  const int row = tid;
  const int qpos = first_qpos + row / NREP;
  float m_run = -INFINITY, l_run = 0.f;
  bool ok = true;

  for (int j = 0; j < n_tiles && ok; ++j) {
    if (tid == 0) {  // S = Q K_j^T
      bool w = (j > 0 || mbar_wait(&bar_q, 0)) && mbar_wait(&bar_kv[j & 1], (j >> 1) & 1);
      if (!w) {
        fail_s = 1;
      } else {
        consumed = j + 1;
        fence_after();
        const unsigned char* kt = kv_s + (j & 1) * kStageBytes;
#pragma unroll
        for (int k = 0; k < kD / 16; ++k) {
          const int h = k >> 2, off = (k & 3) * 32;
          umma<false>(t_S, desc_kmajor(q_s + h * kHalf + off), desc_kmajor(kt + h * kHalf + off), k > 0 ? 1u : 0u);
        }
        mma_commit(&bar_s);
      }
    }
    // every thread: wait for S
    if (!__all_sync(0xffffffffu, mbar_wait(&bar_s, j & 1))) {
      if (lane == 0) fail_s = 1;
    }
    __syncthreads();
    if (fail_s) {
      ok = false;
      break;
    }
    fence_after();
    // pass 1: row max of the masked, scaled scores
    const int key0 = j * kKeys;
    const bool full = key0 + kKeys - 1 <= first_qpos;  // no key of the tile is masked for any row
    float mx = -INFINITY;
#pragma unroll 1
    for (int c = 0; c < kKeys; c += 32) {
      float v[32];
      tmem_ld32(t_S + lane_base + c, v);
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const bool valid = full || key0 + c + i <= qpos;
        mx = fmaxf(mx, valid ? v[i] * p.qscale : -INFINITY);
      }
    }
    const float m_new = fmaxf(m_run, mx);
    const float alpha = m_run == -INFINITY ? 0.f : exp2f(m_run - m_new);
    // pass 2: p = 2^(s - m_new) -> bf16 P row (swizzled K-major), row sum
    float sum = 0.f;
#pragma unroll 1
    for (int c = 0; c < kKeys; c += 32) {
      float v[32];
      tmem_ld32(t_S + lane_base + c, v);
      uint32_t pk[16];
#pragma unroll
      for (int i = 0; i < 32; i += 2) {
        const bool v0 = full || key0 + c + i <= qpos, v1 = full || key0 + c + i + 1 <= qpos;
        const float p0 = v0 ? exp2f(v[i] * p.qscale - m_new) : 0.f;
        const float p1 = v1 ? exp2f(v[i + 1] * p.qscale - m_new) : 0.f;
        sum += p0 + p1;
        const __nv_bfloat162 b = __floats2bfloat162_rn(p0, p1);
        pk[i / 2] = *reinterpret_cast<const uint32_t*>(&b);
      }
      unsigned char* prow = p_s + (c >> 6) * kHalf + row * 128;
#pragma unroll
      for (int ch = 0; ch < 4; ++ch) {  // 4 chunks of 8 keys
        const int chunk = ((c & 63) >> 3) + ch;
        *reinterpret_cast<uint4*>(prow + ((chunk ^ (row & 7)) << 4)) =
            make_uint4(pk[4 * ch], pk[4 * ch + 1], pk[4 * ch + 2], pk[4 * ch + 3]);
      }
    }
    l_run = l_run * alpha + sum;
    m_run = m_new;
    // O of the previous tile must be complete before it is rescaled and before P is reused
    if (j > 0) {
      if (!__all_sync(0xffffffffu, mbar_wait(&bar_o, (j - 1) & 1))) {
        if (lane == 0) fail_s = 1;
      }
      fence_after();
      if (__any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll 1
        for (int c = 0; c < kD; c += 32) {
          float v[32];
          tmem_ld32(t_O + lane_base + c, v);
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] *= alpha;
          tmem_st32(t_O + lane_base + c, v);
        }
      }
      if (tid == 0 && j + 1 < n_tiles) {  // its stage held tile j - 1, now consumed
        load_kv(j + 1);
        issued = j + 2;
      }
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // P: generic writes -> MMA reads
    fence_before();
    __syncthreads();
    if (fail_s) {
      ok = false;
      break;
    }
    if (tid == 0) {  // O += P V_j
      fence_after();
      const unsigned char* vt = kv_s + (j & 1) * kStageBytes + kTileBytes;
#pragma unroll
      for (int k = 0; k < kKeys / 16; ++k) {
        const int h = k >> 2, off = (k & 3) * 32;
        umma<true>(t_O, desc_kmajor(p_s + h * kHalf + off), desc_mnmajor(vt + k * 16 * 128),
                   (j > 0 || k > 0) ? 1u : 0u);
      }
      mma_commit(&bar_o);
    }
  }

  // epilogue: O / l -> bf16 rows
  const bool done = ok && __all_sync(0xffffffffu, mbar_wait(&bar_o, (n_tiles - 1) & 1));
  if (!done) {
    if (lane == 0) atomicOr(p.err, 4);
  } else {
    fence_after();
    const int pos = q0 + row / NREP;
    const int head = kvh * NREP + row % NREP;
    const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
    __nv_bfloat16* dst = p.out + ((int64_t)(tok0 + pos) * p.H + head) * kD;
#pragma unroll 1
    for (int c = 0; c < kD; c += 32) {
      float v[32];
      tmem_ld32(t_O + lane_base + c, v);
      if (pos < qlen) {
#pragma unroll
        for (int i = 0; i < 32; i += 8) {
          __nv_bfloat162 a = __floats2bfloat162_rn(v[i] * inv, v[i + 1] * inv);
          __nv_bfloat162 b = __floats2bfloat162_rn(v[i + 2] * inv, v[i + 3] * inv);
          __nv_bfloat162 cc = __floats2bfloat162_rn(v[i + 4] * inv, v[i + 5] * inv);
          __nv_bfloat162 d = __floats2bfloat162_rn(v[i + 6] * inv, v[i + 7] * inv);
          uint4 w;
          w.x = *reinterpret_cast<uint32_t*>(&a); w.y = *reinterpret_cast<uint32_t*>(&b);
          w.z = *reinterpret_cast<uint32_t*>(&cc); w.w = *reinterpret_cast<uint32_t*>(&d);
          *reinterpret_cast<uint4*>(dst + c + i) = w;
        }
      }
    }
  }
  if (tid == 0 && !ok) {  // let issued copies land before the CTA exits (bounded)
    (void)mbar_wait(&bar_q, 0);
    for (int t = consumed; t < issued; ++t) (void)mbar_wait(&bar_kv[t & 1], (t >> 1) & 1);
    atomicOr(p.err, 4);
  }
  fence_before();
  __syncthreads();
  if (warp == 0) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(256));
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
  static unsigned configured = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 32 && !(configured & (1u << dev))) {
    cudaFuncSetAttribute(prefill_tc_kernel<NREP>, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    configured |= 1u << dev;
  }
  prefill_tc_kernel<NREP><<<dim3(p.n_kv, items), 128, kSmemBytes, st>>>(tq, tk, tv, p);
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
