// Batch-metadata buffer layout shared by the meta builder, the attention
// kernels and the forward orchestration.
#pragma once

#include "common.cuh"

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

// qp: query positions per multi-token attention tile (see query_tile_positions).
// pool: persistent block-table pool [pool_slots][L.W_cap] for records in the
// pooled layout (NULL for records that carry their tables).
int build_batch_meta(const int32_t* rec, const MetaLayout& L, int bs, int num_blocks, int qp,
                     int32_t* meta, cudaStream_t st, int32_t* pool = nullptr, int pool_slots = 0);

}  // namespace vllt
