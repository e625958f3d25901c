// Device code of the generic varlen paged attention (launched by
// attention.cu): attention_kernel and the split-K merge. Plain CUDA C++ with
// no inline PTX beyond device_common.cuh's helpers, so the CPU tests can also
// run it on the host (tests/simt_host.h).
#pragma once

#include <math.h>
#include <stddef.h>
#include <stdint.h>

#include "device_common.cuh"

namespace vllt {
namespace ak {

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

  VLLT_DYNAMIC_SMEM(smem_raw, 16);
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

// Dynamic shared memory of one attention_kernel launch: the staging layout,
// or the warps' merge state (which reuses the staging area after q_s) if larger.
template <typename T, int D, int ROWS>
size_t attention_smem_bytes() {
  const size_t merge = sizeof(float) * (2 * kWarps * ROWS + kWarps * ROWS * D) + sizeof(float) * ROWS * D;
  return attention_smem<T, D, ROWS>() > merge ? attention_smem<T, D, ROWS>() : merge;
}

}  // namespace ak
}  // namespace vllt
