// Device code of the batch-flatten kernel (launched by batch_meta.cu). Plain
// CUDA C++ with no inline PTX, so the CPU tests can also run it on the host
// (tests/simt_host.h).
#pragma once

#include <stdint.h>

#include "device_common.cuh"
#include "meta_items.cuh"

namespace vllt {
namespace bmk {

constexpr int kThreads = 1024;

// Block-wide exclusive scan of an int4 (four independent counters).
__device__ int4 block_exclusive_scan(int4 v, int4* warp_tot, int4* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int4 incl = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int4 n;
    n.x = __shfl_up_sync(0xffffffffu, incl.x, o);
    n.y = __shfl_up_sync(0xffffffffu, incl.y, o);
    n.z = __shfl_up_sync(0xffffffffu, incl.z, o);
    n.w = __shfl_up_sync(0xffffffffu, incl.w, o);
    if (lane >= o) { incl.x += n.x; incl.y += n.y; incl.z += n.z; incl.w += n.w; }
  }
  if (lane == 31) warp_tot[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int4 t = warp_tot[lane];
    int4 it = t;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int4 n;
      n.x = __shfl_up_sync(0xffffffffu, it.x, o);
      n.y = __shfl_up_sync(0xffffffffu, it.y, o);
      n.z = __shfl_up_sync(0xffffffffu, it.z, o);
      n.w = __shfl_up_sync(0xffffffffu, it.w, o);
      if (lane >= o) { it.x += n.x; it.y += n.y; it.z += n.z; it.w += n.w; }
    }
    warp_tot[lane] = make_int4(it.x - t.x, it.y - t.y, it.z - t.z, it.w - t.w);
    if (lane == 31) *total = it;
  }
  __syncthreads();
  int4 base = warp_tot[warp];
  int4 r = make_int4(base.x + incl.x - v.x, base.y + incl.y - v.y, base.z + incl.z - v.z,
                     base.w + incl.w - v.w);
  __syncthreads();
  return r;
}

// `pool` (NULL: the record carries the tables) is the persistent block-table
// pool [pool_slots][L.W_cap]: the record then carries, after the tokens, each
// sequence's pool slot and a list of (slot, index, block id) updates that
// this kernel applies to the pool before it reads the tables through the
// slots (the record layout is in include/vllt.h). Token ids are resolved
// against `tsrc` (the previous pass's picks, tsrc_len entries; may be NULL)
// and checked against the embedding's `vocab` rows.
__global__ void __launch_bounds__(kThreads) build_meta_kernel(const int32_t* __restrict__ rec,
                                                              MetaLayout L, int bs, int num_blocks,
                                                              int qp, int32_t* __restrict__ meta,
                                                              int32_t* __restrict__ pool, int pool_slots,
                                                              const int32_t* __restrict__ tsrc, int tsrc_len,
                                                              int vocab) {
  __shared__ int4 warp_tot[32];
  __shared__ int4 total;
  // s_err: errors that stop the step (read by every thread right after phase
  // 1); s_err_run: errors of phases 2-3 that leave it runnable. Two words,
  // so no thread can change the first while a slower warp still reads it.
  __shared__ int s_max_ctx, s_max_q, s_err, s_err_run;
  const int S = rec[0], T = rec[1], R = rec[2], W = rec[3];
  const int U = pool ? rec[4] : 0;  // pool updates carried by this record
  int32_t* cnt = meta;
  const bool fits = S >= 0 && T >= 0 && R >= 0 && W >= 0 && S <= L.S_cap && T <= L.T_cap &&
                    R <= L.R_cap && W <= L.W_cap && U >= 0 && (int64_t)U <= (int64_t)L.S_cap * L.W_cap;
  if (!fits) {  // uniform across the CTA: every thread takes this branch
    if (threadIdx.x == 0) {
      for (int i = 0; i < kCntWords; ++i) cnt[i] = 0;
      cnt[kCntError] = 1;
    }
    return;
  }
  const int32_t* start = rec + (pool ? 5 : 4);
  const int32_t* qlen = start + S;
  const int32_t* count = qlen + S;
  const int32_t* tokens = count + S;
  const int32_t* tables = tokens + T;       // record tables [S][W] (no pool)
  const int32_t* seq_slot = tokens + T;     // pool slot of each sequence (pool)
  const int32_t* updates = seq_slot + S;    // [U][3] (slot, index, block) (pool)
  int32_t* cu_q = meta + L.cu_q;
  int32_t* cu_rows = meta + L.cu_rows;
  int32_t* ctx = meta + L.ctx;
  int32_t* mstart = meta + L.start;
  if (threadIdx.x == 0) { s_max_ctx = 0; s_max_q = 0; s_err = 0; s_err_run = 0; }
  __syncthreads();

  // Phase 0 (pool): apply this pass's block-table changes. An update outside
  // the pool flags the step (bit 1) and is dropped.
  for (int u = threadIdx.x; u < U; u += kThreads)
    if (!pool_update(pool, pool_slots, L.W_cap, updates + 3 * u)) atomicOr(&s_err, 2);
  __syncthreads();  // the pool writes above are visible to every thread of the CTA below

  // Phase 1: exclusive scans over sequences of (qlen, count, is_decode, tiles).
  int32_t* cu_tiles = meta + L.cu_tiles;
  int4 carry = make_int4(0, 0, 0, 0);
  for (int base = 0; base < S; base += kThreads) {
    const int s = base + threadIdx.x;
    int4 v = make_int4(0, 0, 0, 0);
    if (s < S) {
      const int q = qlen[s];
      v = make_int4(q, count[s], q == 1 ? 1 : 0, seq_tiles(q, qp));
      atomicMax(&s_max_ctx, start[s] + q);
      atomicMax(&s_max_q, q);
      if (seq_fields_bad(start[s], q, count[s], W, bs)) atomicOr(&s_err, 2);
    }
    int4 ex = block_exclusive_scan(v, warp_tot, &total);
    if (s < S) {
      cu_q[s] = carry.x + ex.x;
      cu_rows[s] = carry.y + ex.y;
      ctx[s] = start[s] + qlen[s];
      mstart[s] = start[s];
      cu_tiles[s] = carry.w + ex.w;
      if (v.z) meta[L.dec_seq + carry.z + ex.z] = s;
    }
    carry.x += total.x; carry.y += total.y; carry.z += total.z; carry.w += total.w;
  }
  if (threadIdx.x == 0) {
    cu_q[S] = carry.x;
    cu_rows[S] = carry.y;
    cu_tiles[S] = carry.w;
    if (carry.x != T || carry.y != R || carry.w > L.tiles_cap) atomicOr(&s_err, 1);
  }
  __syncthreads();
  if (s_err) {  // uniform: nothing downstream may index with inconsistent counts
    if (threadIdx.x == 0) {
      for (int i = 0; i < kCntWords; ++i) cnt[i] = 0;
      cnt[kCntError] = s_err;
    }
    return;
  }

  // Phase 2: block tables into the fixed-width copy, validated. From the pool,
  // only the entries a sequence's context uses are read (the rest of a pool
  // row may hold a previous owner's ids); the others become -1.
  for (int i = threadIdx.x; i < S * W; i += kThreads) {
    const int s = i / W, b = i % W;
    const int used = ceil_div(ctx[s], bs);
    int blk;
    if (pool) {
      bool bad = false;
      blk = pool_entry(pool, pool_slots, L.W_cap, seq_slot[s], b, used, num_blocks, &bad);
      if (bad) atomicOr(&s_err_run, 2);
    } else {
      bool bad = false;
      blk = record_entry(tables[i], b, used, num_blocks, &bad);
      if (bad) atomicOr(&s_err_run, 2);
    }
    meta[L.tables + (int64_t)s * L.W_cap + b] = blk;
  }
  __syncthreads();

  // Phase 3: per token -> sequence, position, flat slot (runner.py:75, :83-84).
  const int Tv = min(T, cu_q[S]);
  for (int t = threadIdx.x; t < Tv; t += kThreads) {
    const TokenMeta m = token_meta(cu_q, S, start, meta + L.tables, L.W_cap, W, bs, t);
    meta[L.pos + t] = m.pos;
    meta[L.tok_seq + t] = m.seq;
    bool bad = false;
    meta[L.tokens + t] = resolve_token(tokens[t], tsrc, tsrc_len, vocab, &bad);
    if (bad) atomicOr(&s_err_run, 2);
    meta[L.slot + t] = m.slot;
  }
  // Phase 4: logit rows = the last `count` tokens of each sequence (runner.py:86-90).
  const int Rv = min(R, cu_rows[S]);
  for (int r = threadIdx.x; r < Rv; r += kThreads) meta[L.rows + r] = row_token(cu_rows, cu_q, qlen, count, S, r);
  // Phase 5: multi-token query tiles (seq, first query index).
  const int n_tiles = cu_tiles[S];
  for (int i = threadIdx.x; i < n_tiles; i += kThreads) {
    const int s = upper_index(cu_tiles, S + 1, i);
    meta[L.tile_seq + i] = s;
    meta[L.tile_q0 + i] = (i - cu_tiles[s]) * qp;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    cnt[kCntSeqs] = S;
    cnt[kCntTokens] = T;
    cnt[kCntRows] = R;
    cnt[kCntWidth] = W;
    cnt[kCntDecode] = carry.z;
    cnt[kCntTiles] = carry.w;
    cnt[kCntMaxCtx] = s_max_ctx;
    cnt[kCntMaxQlen] = s_max_q;
    cnt[kCntError] = s_err_run;  // table / token errors (bit 1) leave the step runnable: slots are -1
  }
}

}  // namespace bmk
}  // namespace vllt
