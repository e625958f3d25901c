// Varlen causal paged attention (decode, chunked prefill, speculative verify).
//
// Restates paged_attention (vllmlite/attention.py:59-98) for a whole ragged
// batch in one launch instead of the per-sequence loop at
// vllmlite/model.py:105-112:
//   * query j of sequence s sits at position ctx_s - qlen_s + j and sees keys
//     0..that position (attention.py:70-72, :87-94);
//   * query head h reads KV head h / n_rep; the n_rep heads of one KV head are
//     folded into the rows of one CTA so each K/V tile is read once per group
//     (attention.py:80-84);
//   * scores = (q . k) * scale, softmax, then P @ V (attention.py:84-97), done
//     as an online softmax in fp32.
//
// Work decomposition. A CTA owns one work item (sequence, first query) x one
// KV head. Its rows are (query position, head-in-group) pairs, position-major.
// The 4 warps split the key range: warp w takes 32-key tiles w, w+4, ... and
// keeps a private running (max, sum, acc) per row; the four partial states are
// merged through shared memory at the end. Optionally the key range is also
// split across CTAs (grid.z, "split-K") with a merge kernel, for long contexts
// with few queries.
//
// Staging. Each warp copies its 32 keys' K and V rows into shared memory with
// 16-byte cp.async (zero-filled past the end). One block of one KV head is a
// contiguous bs x D tile in the cache, so consecutive keys of a block are
// consecutive rows. Rows are padded by 16 bytes so the float4 reads of the
// score loop are bank-conflict free.

#include <math.h>

#include <algorithm>

#include "ops.cuh"

namespace vllt {

namespace {

constexpr int kWarps = 4;
constexpr int kKeys = 32;  // keys per warp tile

struct AttnParams {
  const void* q;       // [T][H][D]
  const void* kc;      // [NB][n_kv][bs][D]
  const void* vc;
  void* out;           // [T][H][D]
  const int32_t* tables;  // [S][W]
  int W;
  const int32_t* cu_q;    // [S+1]
  const int32_t* ctx;     // [S]
  // work items: item_seq/item_q0 arrays with a device count, or (standalone)
  // items_per_seq items per sequence over num_seqs sequences.
  const int32_t* item_seq;
  const int32_t* item_q0;
  const int32_t* n_items;
  int items_per_seq;
  int num_seqs;
  int qp;  // query positions per item
  int H, n_kv, n_rep, bs, num_blocks;
  float scale;
  // split-K
  int split_len;      // keys per split (multiple of kWarps*kKeys); 0 = no split
  float* ws_o;        // [splits][P_cap][H][D]  (P_cap = sequence capacity)
  float* ws_ml;       // [splits][P_cap][H][2]
  int P_cap;
};

template <typename T, int D>
struct Tile {
  static constexpr int kPad = 16 / sizeof(T);
  static constexpr int kStride = D + kPad;  // elements per staged row
};

template <typename T, int D, int ROWS>
__global__ void __launch_bounds__(kWarps * 32) attention_kernel(AttnParams p) {
  static_assert((D * sizeof(T)) % 16 == 0, "row must be whole 16-byte chunks");
  constexpr int DI = (D + 31) / 32;   // accumulator slots per lane
  constexpr int CH = D / 4;           // 4-element chunks per row
  constexpr int STR = Tile<T, D>::kStride;
  constexpr int VPR = D * (int)sizeof(T) / 16;  // 16-byte vectors per row

  extern __shared__ __align__(16) unsigned char smem_raw[];
  float* q_s = reinterpret_cast<float*>(smem_raw);                       // [ROWS][D]
  T* kv_s = reinterpret_cast<T*>(q_s + ROWS * D);                       // [kWarps][2][32][STR]
  float* p_s = reinterpret_cast<float*>(kv_s + kWarps * 2 * kKeys * STR);  // [kWarps][ROWS][32]

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int kvh = blockIdx.x;
  const int item = blockIdx.y;
  int s, q0;
  if (p.item_seq) {
    if (item >= *p.n_items) return;
    s = p.item_seq[item];
    q0 = p.item_q0 ? p.item_q0[item] : 0;
  } else {
    s = item / p.items_per_seq;
    q0 = (item % p.items_per_seq) * p.qp;
    if (s >= p.num_seqs) return;
  }
  const int tok0 = p.cu_q[s];
  const int qlen = p.cu_q[s + 1] - tok0;
  if (q0 >= qlen) return;
  const int npos = min(p.qp, qlen - q0);
  const int nrows = npos * p.n_rep;
  const int ctx = p.ctx[s];
  const int first_qpos = ctx - qlen + q0;
  const int last_qpos = first_qpos + npos - 1;

  // key range of this CTA
  int k_begin = 0, k_end = min(last_qpos + 1, p.W * p.bs);
  const int split = blockIdx.z;
  if (p.split_len > 0) {
    k_begin = split * p.split_len;
    k_end = min(k_end, k_begin + p.split_len);
  }

  // queries -> shared (fp32)
  const T* qg = reinterpret_cast<const T*>(p.q);
  for (int i = threadIdx.x; i < ROWS * D; i += blockDim.x) {
    const int r = i / D, d = i % D;
    float v = 0.f;
    if (r < nrows) {
      const int jp = r / p.n_rep, rep = r % p.n_rep;
      const int h = kvh * p.n_rep + rep;
      v = to_f32(qg[((int64_t)(tok0 + q0 + jp) * p.H + h) * D + d]);
    }
    q_s[i] = v;
  }
  __syncthreads();

  float m_run[ROWS], l_run[ROWS], acc[ROWS][DI];
#pragma unroll
  for (int r = 0; r < ROWS; ++r) {
    m_run[r] = -INFINITY;
    l_run[r] = 0.f;
#pragma unroll
    for (int i = 0; i < DI; ++i) acc[r][i] = 0.f;
  }

  T* k_s = kv_s + warp * 2 * kKeys * STR;
  T* v_s = k_s + kKeys * STR;
  float* pw = p_s + warp * ROWS * kKeys;
  const T* kc = reinterpret_cast<const T*>(p.kc);
  const T* vc = reinterpret_cast<const T*>(p.vc);
  const int32_t* table = p.tables + (int64_t)s * p.W;

  for (int kt = k_begin + warp * kKeys; kt < k_end; kt += kWarps * kKeys) {
    // stage 32 keys: K and V rows, 16-byte vectors, zero-filled when invalid
    for (int i = lane; i < kKeys * VPR; i += 32) {
      const int j = i / VPR, c = i % VPR;
      const int kp = kt + j;
      bool ok = kp < k_end;
      int64_t src = 0;
      if (ok) {
        const int blk = table[kp / p.bs];
        ok = blk >= 0 && blk < p.num_blocks;
        src = (((int64_t)blk * p.n_kv + kvh) * p.bs + kp % p.bs) * D + c * (16 / (int)sizeof(T));
      }
      const int dst = j * STR + c * (16 / (int)sizeof(T));
      cp_async16(k_s + dst, ok ? (const void*)(kc + src) : (const void*)kc, ok);
      cp_async16(v_s + dst, ok ? (const void*)(vc + src) : (const void*)vc, ok);
    }
    cp_async_commit();
    cp_async_wait<0>();
    __syncwarp();

    // scores: lane j <-> key kt + j
    float sc[ROWS];
#pragma unroll
    for (int r = 0; r < ROWS; ++r) sc[r] = 0.f;
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      const float4 kf = load4(k_s + lane * STR + 4 * c);
#pragma unroll
      for (int r = 0; r < ROWS; ++r) {
        const float4 qf = *reinterpret_cast<const float4*>(q_s + r * D + 4 * c);
        sc[r] = fmaf(qf.x, kf.x, sc[r]);
        sc[r] = fmaf(qf.y, kf.y, sc[r]);
        sc[r] = fmaf(qf.z, kf.z, sc[r]);
        sc[r] = fmaf(qf.w, kf.w, sc[r]);
      }
    }
    const int kp = kt + lane;
#pragma unroll
    for (int r = 0; r < ROWS; ++r) {
      if (r < nrows) {
        const int qpos = first_qpos + r / p.n_rep;
        const float x = (kp < k_end && kp <= qpos) ? sc[r] * p.scale : -INFINITY;
        const float mn = fmaxf(m_run[r], warp_max(x));
        const float pr = x == -INFINITY ? 0.f : expf(x - mn);
        const float alpha = m_run[r] == -INFINITY ? 0.f : expf(m_run[r] - mn);
        l_run[r] = l_run[r] * alpha + warp_sum(pr);
        m_run[r] = mn;
#pragma unroll
        for (int i = 0; i < DI; ++i) acc[r][i] *= alpha;
        pw[r * kKeys + lane] = pr;
      }
    }
    __syncwarp();
    // P @ V: lane owns d = lane + 32 i
    const int jmax = min(kKeys, k_end - kt);
    for (int j = 0; j < jmax; ++j) {
      float vv[DI];
#pragma unroll
      for (int i = 0; i < DI; ++i) {
        const int d = lane + 32 * i;
        vv[i] = (d < D) ? to_f32(v_s[j * STR + d]) : 0.f;
      }
#pragma unroll
      for (int r = 0; r < ROWS; ++r) {
        if (r < nrows) {
          const float pj = pw[r * kKeys + j];
#pragma unroll
          for (int i = 0; i < DI; ++i) acc[r][i] = fmaf(pj, vv[i], acc[r][i]);
        }
      }
    }
    __syncwarp();
  }

  // merge the four warps' partial softmax states (reusing the K/V staging area)
  __syncthreads();
  float* m_s = reinterpret_cast<float*>(kv_s);     // [kWarps][ROWS]
  float* l_s = m_s + kWarps * ROWS;                 // [kWarps][ROWS]
  float* a_s = l_s + kWarps * ROWS;                 // [kWarps][ROWS][D]
  if (lane == 0) {
#pragma unroll
    for (int r = 0; r < ROWS; ++r) {
      m_s[warp * ROWS + r] = m_run[r];
      l_s[warp * ROWS + r] = l_run[r];
    }
  }
#pragma unroll
  for (int r = 0; r < ROWS; ++r) {
#pragma unroll
    for (int i = 0; i < DI; ++i) {
      const int d = lane + 32 * i;
      if (d < D) a_s[(warp * ROWS + r) * D + d] = acc[r][i];
    }
  }
  __syncthreads();
  T* og = reinterpret_cast<T*>(p.out);
  for (int i = threadIdx.x; i < nrows * D; i += blockDim.x) {
    const int r = i / D, d = i % D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) M = fmaxf(M, m_s[w * ROWS + r]);
    float L = 0.f, O = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < kWarps; ++w) {
        const float mw = m_s[w * ROWS + r];
        const float e = mw == -INFINITY ? 0.f : expf(mw - M);
        L = fmaf(l_s[w * ROWS + r], e, L);
        O = fmaf(a_s[(w * ROWS + r) * D + d], e, O);
      }
    }
    const int jp = r / p.n_rep, rep = r % p.n_rep;
    const int h = kvh * p.n_rep + rep;
    const int t = tok0 + q0 + jp;
    if (p.split_len > 0) {
      const int64_t base = ((int64_t)split * p.P_cap + s) * p.H + h;
      p.ws_o[base * D + d] = L > 0.f ? O / L : 0.f;
      if (d == 0) {
        p.ws_ml[base * 2] = M;
        p.ws_ml[base * 2 + 1] = L;
      }
    } else {
      og[((int64_t)t * p.H + h) * D + d] = from_f32<T>(L > 0.f ? O / L : 0.f);
    }
  }
}

// Merge split-K partials of single-query work items: one warp per (item, head).
template <typename T, int D>
__global__ void merge_splits_kernel(AttnParams p, int max_splits) {
  pdl_trigger();  // the o_proj projection may start its set-up (it waits for this grid)
  const int lane = threadIdx.x & 31;
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int item = gw / p.H, h = gw % p.H;
  int s;
  if (p.item_seq) {
    if (item >= *p.n_items) return;
    s = p.item_seq[item];
  } else {
    s = item;
    if (s >= p.num_seqs) return;
  }
  const int t = p.cu_q[s];
  const int nsplit = min(max_splits, ceil_div(p.ctx[s], p.split_len));
  float M = -INFINITY;
  for (int z = 0; z < nsplit; ++z) M = fmaxf(M, p.ws_ml[(((int64_t)z * p.P_cap + s) * p.H + h) * 2]);
  float L = 0.f, O[(D + 31) / 32];
#pragma unroll
  for (int i = 0; i < (D + 31) / 32; ++i) O[i] = 0.f;
  for (int z = 0; z < nsplit; ++z) {
    const int64_t base = ((int64_t)z * p.P_cap + s) * p.H + h;
    const float mz = p.ws_ml[base * 2], lz = p.ws_ml[base * 2 + 1];
    if (mz == -INFINITY) continue;
    const float w = lz * expf(mz - M);
    L += w;
#pragma unroll
    for (int i = 0; i < (D + 31) / 32; ++i) {
      const int d = lane + 32 * i;
      if (d < D) O[i] = fmaf(w, p.ws_o[base * D + d], O[i]);
    }
  }
  T* og = reinterpret_cast<T*>(p.out);
#pragma unroll
  for (int i = 0; i < (D + 31) / 32; ++i) {
    const int d = lane + 32 * i;
    if (d < D) og[((int64_t)t * p.H + h) * D + d] = from_f32<T>(L > 0.f ? O[i] / L : 0.f);
  }
}

template <typename T, int D, int ROWS>
size_t attention_smem() {
  return sizeof(float) * ROWS * D + sizeof(T) * kWarps * 2 * kKeys * Tile<T, D>::kStride +
         sizeof(float) * kWarps * ROWS * kKeys;
}

template <typename T, int D, int ROWS>
int launch_attention(const AttnParams& p, int grid_items, int splits, cudaStream_t st) {
  const size_t smem = std::max(attention_smem<T, D, ROWS>(),
                               sizeof(float) * (2 * kWarps * ROWS + kWarps * ROWS * D) +
                                   sizeof(float) * ROWS * D);
  static PerDeviceOnce smem_opt_in;  // dynamic shared memory above 48 KB, once per device
  smem_opt_in.run([&] {
    cudaFuncSetAttribute(attention_kernel<T, D, ROWS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)smem);
  });
  dim3 grid(p.n_kv, grid_items, splits);
  attention_kernel<T, D, ROWS><<<grid, kWarps * 32, smem, st>>>(p);
  return check_launch("attention");
}

template <typename T, int D>
int dispatch_rows(const AttnParams& p, int rows, int grid_items, int splits, cudaStream_t st) {
  if (rows <= 2) return launch_attention<T, D, 2>(p, grid_items, splits, st);
  if (rows <= 4) return launch_attention<T, D, 4>(p, grid_items, splits, st);
  if (rows <= 8) return launch_attention<T, D, 8>(p, grid_items, splits, st);
  return launch_attention<T, D, 16>(p, grid_items, splits, st);
}

template <typename T>
int dispatch_dim(const AttnParams& p, int D, int rows, int grid_items, int splits, cudaStream_t st) {
  switch (D) {
    case 8: return dispatch_rows<T, 8>(p, rows, grid_items, splits, st);
    case 16: return dispatch_rows<T, 16>(p, rows, grid_items, splits, st);
    case 32: return dispatch_rows<T, 32>(p, rows, grid_items, splits, st);
    case 48: return dispatch_rows<T, 48>(p, rows, grid_items, splits, st);
    case 64: return dispatch_rows<T, 64>(p, rows, grid_items, splits, st);
    case 128: return dispatch_rows<T, 128>(p, rows, grid_items, splits, st);
    default: set_error("attention: head_dim %d not built (8,16,32,48,64,128)", D); return VLLT_ERR_UNSUPPORTED;
  }
}

template <typename T>
int merge_dim(const AttnParams& p, int D, int items, int splits, cudaStream_t st) {
  if (items <= 0) return VLLT_OK;
  const int warps = items * p.H;
  const int blocks = ceil_div(warps * 32, 256);
  switch (D) {
    case 8: merge_splits_kernel<T, 8><<<blocks, 256, 0, st>>>(p, splits); break;
    case 16: merge_splits_kernel<T, 16><<<blocks, 256, 0, st>>>(p, splits); break;
    case 32: merge_splits_kernel<T, 32><<<blocks, 256, 0, st>>>(p, splits); break;
    case 48: merge_splits_kernel<T, 48><<<blocks, 256, 0, st>>>(p, splits); break;
    case 64: merge_splits_kernel<T, 64><<<blocks, 256, 0, st>>>(p, splits); break;
    case 128: merge_splits_kernel<T, 128><<<blocks, 256, 0, st>>>(p, splits); break;
    default: return VLLT_ERR_UNSUPPORTED;
  }
  return check_launch("attention merge");
}

}  // namespace

// Keys per split-K chunk of the generic kernel.
constexpr int kSplitLen = 512;
constexpr int64_t kFlagBytes = 256;  // attention workspace header: device error word

int64_t decode_ws_bytes(int P_cap, int H, int max_ctx);
bool decode_supported(const AttnCall& c);
int decode_pass(const AttnCall& c, const int32_t* item_seq, const int32_t* n_items, int items_cap, int num_seqs,
                int max_ctx, int* err, cudaStream_t st,
                int (*merge)(const AttnCall&, const int32_t*, const int32_t*, int, int, int, cudaStream_t));

int64_t attention_ws_bytes(int P_cap, int H, int D, int max_ctx) {
  const int splits = ceil_div(max_ctx, kSplitLen);
  const int64_t generic = splits <= 1 ? 0 : (int64_t)splits * P_cap * H * (D + 2) * sizeof(float);
  const int64_t dec = D == 128 ? decode_ws_bytes(P_cap, H, max_ctx) : 0;
  return kFlagBytes + std::max(generic, dec);
}

namespace {

AttnParams params_of(const AttnCall& c) {
  AttnParams p{};
  p.q = c.q; p.kc = c.kc; p.vc = c.vc; p.out = c.out;
  p.tables = c.tables; p.W = c.W; p.cu_q = c.cu_q; p.ctx = c.ctx;
  p.H = c.H; p.n_kv = c.n_kv; p.n_rep = c.H / c.n_kv; p.bs = c.bs; p.num_blocks = c.num_blocks;
  p.scale = c.scale; p.P_cap = c.P_cap;
  return p;
}

// Merge of the decode kernel's splits (1024-token chunks), workspace after the flags header.
int merge_decode_splits(const AttnCall& c, const int32_t* item_seq, const int32_t* n_items, int items,
                        int num_seqs, int splits, cudaStream_t st) {
  AttnParams p = params_of(c);
  p.item_seq = item_seq;
  p.n_items = n_items;
  p.num_seqs = num_seqs;
  p.split_len = 1024;
  p.ws_o = c.ws;
  p.ws_ml = c.ws + (int64_t)splits * c.P_cap * c.H * c.D;
  return c.dtype == VLLT_F32 ? merge_dim<float>(p, c.D, items, splits, st)
                             : merge_dim<__nv_bfloat16>(p, c.D, items, splits, st);
}

}  // namespace

// Shared entry for the forward pass and the C ABI.
//  single-query pass: items = sequences with one query token (item_seq = dec list)
//  tile pass:         items = (seq, q0) tiles
// `c.ws` points at the attention workspace (flags header first) or is NULL.
bool prefill_tc_supported(const AttnCall& c);
int prefill_tc_positions(int n_rep);
int prefill_tc_pass(const AttnCall& c, int T_rows, const int32_t* item_seq, const int32_t* item_q0,
                    const int32_t* n_items, int items_cap, int items_per_seq, int num_seqs, int* err,
                    cudaStream_t st);

int query_tile_positions(int dtype, int head_dim, int block_size, int n_rep) {
  AttnCall c{};
  c.dtype = dtype; c.D = head_dim; c.bs = block_size; c.H = n_rep; c.n_kv = 1;
  return prefill_tc_supported(c) ? prefill_tc_positions(n_rep) : tile_positions(n_rep);
}

int attention_pass(const AttnCall& c0, const int32_t* item_seq, const int32_t* item_q0,
                   const int32_t* n_items, int items_cap, int num_seqs, int max_qlen,
                   bool single_query, int max_ctx, cudaStream_t st) {
  VLLT_REQUIRE(c0.H / c0.n_kv <= 16, "attention: n_heads / n_kv must be <= 16");
  // split the workspace into the flags header and the partials area
  AttnCall c = c0;
  int* flags = nullptr;
  if (c0.ws && c0.ws_bytes >= kFlagBytes) {
    flags = reinterpret_cast<int*>(c0.ws);
    c.ws = reinterpret_cast<float*>(reinterpret_cast<char*>(c0.ws) + kFlagBytes);
    c.ws_bytes = c0.ws_bytes - kFlagBytes;
  } else {
    c.ws = nullptr;
    c.ws_bytes = 0;
  }
  if (c0.err) flags = c0.err;
  const int n_rep = c.H / c.n_kv;
  // standalone: (sequence, tile) items from the batch shape
  int items_per_seq = 1;
  if (!item_seq) {
    const int qp = single_query ? 1 : query_tile_positions(c.dtype, c.D, c.bs, n_rep);
    items_per_seq = single_query ? 1 : ceil_div(std::max(max_qlen, 1), qp);
    VLLT_REQUIRE((int64_t)items_per_seq * num_seqs < (1ll << 31), "attention: too many tiles");
    items_cap = items_per_seq * num_seqs;
  }
  if (items_cap <= 0) return VLLT_OK;
  if (single_query && decode_supported(c) && flags)
    return decode_pass(c, item_seq, n_items, items_cap, num_seqs, max_ctx, flags, st, merge_decode_splits);
  if (!single_query && prefill_tc_supported(c) && flags)
    return prefill_tc_pass(c, c.T_rows, item_seq, item_q0, n_items, items_cap, items_per_seq, num_seqs, flags, st);

  AttnParams p = params_of(c);
  p.item_seq = item_seq; p.item_q0 = item_q0; p.n_items = n_items;
  p.items_per_seq = items_per_seq; p.num_seqs = num_seqs;
  p.qp = single_query ? 1 : tile_positions(p.n_rep);
  const int rows = p.qp * p.n_rep;
  int splits = 1;
  if (single_query && max_ctx > kSplitLen) {
    splits = ceil_div(max_ctx, kSplitLen);
    const int64_t need = (int64_t)splits * c.P_cap * c.H * (c.D + 2) * sizeof(float);
    if (c.ws && c.ws_bytes >= need) {
      p.split_len = kSplitLen;
      p.ws_o = c.ws;
      p.ws_ml = c.ws + (int64_t)splits * c.P_cap * c.H * c.D;
    } else {
      splits = 1;  // no workspace: one CTA walks the whole context
    }
  }
  int rc = c.dtype == VLLT_F32 ? dispatch_dim<float>(p, c.D, rows, items_cap, splits, st)
                               : dispatch_dim<__nv_bfloat16>(p, c.D, rows, items_cap, splits, st);
  if (rc != VLLT_OK || splits == 1) return rc;
  return c.dtype == VLLT_F32 ? merge_dim<float>(p, c.D, items_cap, splits, st)
                             : merge_dim<__nv_bfloat16>(p, c.D, items_cap, splits, st);
}

}  // namespace vllt
