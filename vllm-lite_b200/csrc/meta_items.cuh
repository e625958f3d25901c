// The batch-metadata buffer's layout and the per-item arithmetic of its
// builder (build_meta_kernel, batch_meta.cu): plain integer code with no CUDA
// dependency, shared by the kernel and the host-compiled CPU tests, which run
// these exact functions on the reference's step records.
#pragma once

#include <stdint.h>

#ifndef __CUDACC__
#ifndef __host__
#define __host__
#endif
#ifndef __device__
#define __device__
#endif
#endif

namespace vllt {

// Counter words at the start of the meta buffer.
enum MetaCounter {
  kCntSeqs = 0,     // S
  kCntTokens = 1,   // T
  kCntRows = 2,     // R (logit rows)
  kCntWidth = 3,    // block-table width of the step record
  kCntDecode = 4,   // sequences with exactly one query token
  kCntTiles = 5,    // multi-token query tiles
  kCntMaxCtx = 6,   // longest context this pass
  kCntError = 7,    // nonzero when validation failed (bit 0: capacity, bit 1: table)
  kCntMaxQlen = 8,
  kCntWords = 16
};

// Fixed-capacity layout, in int32 words, so a captured graph's pointers stay
// valid for every step that fits.
struct MetaLayout {
  int S_cap, T_cap, R_cap, W_cap, tiles_cap;
  int64_t cu_q, cu_rows, cu_tiles, ctx, start, pos, slot, tok_seq, tokens, rows, dec_seq, tile_seq,
      tile_q0, tables, words;

  __host__ __device__ static MetaLayout make(int S_cap, int T_cap, int R_cap, int W_cap) {
    MetaLayout L;
    L.S_cap = S_cap;
    L.T_cap = T_cap;
    L.R_cap = R_cap;
    L.W_cap = W_cap;
    L.tiles_cap = T_cap + S_cap;
    int64_t o = kCntWords;
    auto take = [&](int64_t n) { int64_t r = o; o += (n + 3) / 4 * 4; return r; };
    L.cu_q = take(S_cap + 1);
    L.cu_rows = take(S_cap + 1);
    L.cu_tiles = take(S_cap + 1);
    L.ctx = take(S_cap);
    L.start = take(S_cap);
    L.pos = take(T_cap);
    L.slot = take(T_cap);
    L.tok_seq = take(T_cap);
    L.tokens = take(T_cap);
    L.rows = take(R_cap);
    L.dec_seq = take(S_cap);
    L.tile_seq = take(L.tiles_cap);
    L.tile_q0 = take(L.tiles_cap);
    L.tables = take((int64_t)S_cap * W_cap);
    L.words = o;
    return L;
  }
};

// Query positions per multi-token attention tile for a GQA group of n_rep:
// a tile holds up to 16 (position, head) rows.
__host__ __device__ inline int tile_positions(int n_rep) { return n_rep >= 16 ? 1 : 16 / n_rep; }

// Largest i in [0, n) with a[i] <= key (a ascending, a[0] == 0 <= key).
__host__ __device__ inline int upper_index(const int32_t* a, int n, int key) {
  int lo = 0, hi = n - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (a[mid] <= key) lo = mid; else hi = mid - 1;
  }
  return lo;
}

// Phase 1: a sequence's record fields the runner could not index with
// (error bit 1): no query token, a logit-row count outside [1, qlen], a
// negative start, or a context beyond its table's W blocks.
__host__ __device__ inline bool seq_fields_bad(int start, int qlen, int count, int W, int bs) {
  return qlen < 1 || count < 1 || count > qlen || start < 0 || start + qlen > W * bs;
}

// Phase 1: multi-token query tiles of a sequence (qp positions each; a
// single-query sequence is a decode item instead).
__host__ __device__ inline int seq_tiles(int qlen, int qp) { return qlen > 1 ? (qlen + qp - 1) / qp : 0; }

// Phase 0: one (pool row, table index, block id) update into the pool
// [pool_slots][width]; false, with nothing written, when it lies outside.
__host__ __device__ inline bool pool_update(int32_t* pool, int pool_slots, int width, const int32_t* upd) {
  const int row = upd[0], j = upd[1];
  if (row < 0 || row >= pool_slots || j < 0 || j >= width) return false;
  pool[(int64_t)row * width + j] = upd[2];
  return true;
}

// Phase 2, pooled record: entry b of a sequence's block table, read through
// its pool row, for a context that uses `used` blocks: -1 past them (never
// read); -1 with *bad set when the row or the block id is out of range.
__host__ __device__ inline int pool_entry(const int32_t* pool, int pool_slots, int width, int row, int b, int used,
                                          int num_blocks, bool* bad) {
  if (b >= used) return -1;
  int blk = -1;
  if (row >= 0 && row < pool_slots) blk = pool[(int64_t)row * width + b];
  if (blk < 0 || blk >= num_blocks) {
    *bad = true;
    return -1;
  }
  return blk;
}

// Phase 2, classic record: entry b as the record carries it; an id the
// context uses that lies outside [0, num_blocks) becomes -1 with *bad set.
__host__ __device__ inline int record_entry(int blk, int b, int used, int num_blocks, bool* bad) {
  if (b < used && (blk < 0 || blk >= num_blocks)) {
    *bad = true;
    return -1;
  }
  return blk;
}

// Phase 3: query token t -> its sequence, position (runner.py:75:
// start .. start + qlen - 1) and flat cache slot (gather_slots,
// attention.py:40-44), -1 when its block is unknown. `tables` is the
// fixed-width copy [S][table_stride] built in phase 2.
struct TokenMeta {
  int seq, pos, slot;
};
__host__ __device__ inline TokenMeta token_meta(const int32_t* cu_q, int S, const int32_t* start,
                                                const int32_t* tables, int64_t table_stride, int W, int bs, int t) {
  TokenMeta m;
  m.seq = upper_index(cu_q, S + 1, t);
  m.pos = start[m.seq] + (t - cu_q[m.seq]);
  const int b = m.pos / bs;  // pos >= 0 and pos < W * bs were validated in phase 1
  const int blk = b < W ? tables[(int64_t)m.seq * table_stride + b] : -1;
  m.slot = blk < 0 ? -1 : blk * bs + m.pos % bs;
  return m;
}

// Phase 3: the token id a record entry stands for. t >= 0 is the id; t < 0
// is entry -t - 1 of the previous pass's picks (src, src_len entries). An id
// outside [0, vocab) after that, or a reference outside src, is flagged
// (*bad) and yields token 0, so the embedding never reads outside its table.
__host__ __device__ inline int resolve_token(int32_t t, const int32_t* src, int src_len, int vocab, bool* bad) {
  if (t < 0) {
    const int64_t i = -(int64_t)t - 1;
    if (!src || i >= src_len) {
      *bad = true;
      return 0;
    }
    t = src[i];
  }
  if (t < 0 || t >= vocab) {
    *bad = true;
    return 0;
  }
  return t;
}

// Phase 4: logit row r -> its query token: the last `count` tokens of each
// sequence (runner.py:86-90).
__host__ __device__ inline int row_token(const int32_t* cu_rows, const int32_t* cu_q, const int32_t* qlen,
                                         const int32_t* count, int S, int r) {
  const int s = upper_index(cu_rows, S + 1, r);
  return cu_q[s] + qlen[s] - count[s] + (r - cu_rows[s]);
}

}  // namespace vllt
