// Test harness: build_meta_kernel (csrc/batch_meta.cu) with its per-item
// arithmetic (csrc/meta_items.cuh) compiled for the host; the phases run one
// after another, the block-wide scans as plain running sums. Built by the CPU
// tests with g++ (tests/host_build.py).
#include "meta_items.cuh"

using namespace vllt;

// Phases 0 and 2 of a pooled step record: applies its updates to `pool` and
// writes each sequence's table [S][W] as the kernel reads it; returns the
// kernel's error bits.
extern "C" int apply_pooled_host(const int32_t* rec, int32_t* pool, int pool_slots, int width, int block_size,
                                 int num_blocks, int32_t* tables) {
  const int S = rec[0], T = rec[1], W = rec[3], U = rec[4];
  const int32_t* start = rec + 5;
  const int32_t* qlen = start + S;
  const int32_t* slot = qlen + 2 * S + T;  // after counts and tokens
  const int32_t* updates = slot + S;
  int err = 0;
  for (int u = 0; u < U; ++u)
    if (!pool_update(pool, pool_slots, width, updates + 3 * u)) err |= 2;
  for (int s = 0; s < S; ++s) {
    const int used = (start[s] + qlen[s] + block_size - 1) / block_size;
    for (int b = 0; b < W; ++b) {
      bool bad = false;
      tables[s * W + b] = pool_entry(pool, pool_slots, width, slot[s], b, used, num_blocks, &bad);
      if (bad) err |= 2;
    }
  }
  return err;
}

// The whole metadata buffer (MetaLayout of the capacities) of one step
// record, classic (pool == NULL) or pooled, with record token ids resolved
// against tsrc (may be NULL) and checked against vocab; returns the error word.
extern "C" int build_meta_host(const int32_t* rec, int32_t* pool, int pool_slots, int S_cap, int T_cap, int R_cap,
                               int W_cap, int bs, int num_blocks, int qp, int32_t* meta, const int32_t* tsrc,
                               int tsrc_len, int vocab) {
  const MetaLayout L = MetaLayout::make(S_cap, T_cap, R_cap, W_cap);
  const int S = rec[0], T = rec[1], R = rec[2], W = rec[3];
  const int U = pool ? rec[4] : 0;
  int32_t* cnt = meta;
  const bool fits = S >= 0 && T >= 0 && R >= 0 && W >= 0 && S <= L.S_cap && T <= L.T_cap && R <= L.R_cap &&
                    W <= L.W_cap && U >= 0 && (int64_t)U <= (int64_t)L.S_cap * L.W_cap;
  if (!fits) {
    for (int i = 0; i < kCntWords; ++i) cnt[i] = 0;
    return cnt[kCntError] = 1;
  }
  const int32_t* start = rec + (pool ? 5 : 4);
  const int32_t* qlen = start + S;
  const int32_t* count = qlen + S;
  const int32_t* tokens = count + S;
  const int32_t* tables = tokens + T;
  const int32_t* seq_slot = tokens + T;
  const int32_t* updates = seq_slot + S;
  int32_t *cu_q = meta + L.cu_q, *cu_rows = meta + L.cu_rows, *cu_tiles = meta + L.cu_tiles, *ctx = meta + L.ctx;
  int err = 0;
  for (int u = 0; u < U; ++u)  // phase 0
    if (!pool_update(pool, pool_slots, L.W_cap, updates + 3 * u)) err |= 2;
  int cq = 0, cr = 0, cd = 0, ct = 0, max_ctx = 0, max_q = 0;  // phase 1
  for (int s = 0; s < S; ++s) {
    const int q = qlen[s];
    cu_q[s] = cq;
    cu_rows[s] = cr;
    cu_tiles[s] = ct;
    ctx[s] = start[s] + q;
    meta[L.start + s] = start[s];
    if (q == 1) meta[L.dec_seq + cd++] = s;
    cq += q;
    cr += count[s];
    ct += seq_tiles(q, qp);
    if (start[s] + q > max_ctx) max_ctx = start[s] + q;
    if (q > max_q) max_q = q;
    if (seq_fields_bad(start[s], q, count[s], W, bs)) err |= 2;
  }
  cu_q[S] = cq;
  cu_rows[S] = cr;
  cu_tiles[S] = ct;
  if (cq != T || cr != R || ct > L.tiles_cap) err |= 1;
  if (err) {
    for (int i = 0; i < kCntWords; ++i) cnt[i] = 0;
    return cnt[kCntError] = err;
  }
  for (int s = 0; s < S; ++s) {  // phase 2
    const int used = (ctx[s] + bs - 1) / bs;
    for (int b = 0; b < W; ++b) {
      bool bad = false;
      const int blk = pool ? pool_entry(pool, pool_slots, L.W_cap, seq_slot[s], b, used, num_blocks, &bad)
                           : record_entry(tables[s * W + b], b, used, num_blocks, &bad);
      if (bad) err |= 2;
      meta[L.tables + (int64_t)s * L.W_cap + b] = blk;
    }
  }
  for (int t = 0; t < T && t < cu_q[S]; ++t) {  // phase 3
    const TokenMeta m = token_meta(cu_q, S, start, meta + L.tables, L.W_cap, W, bs, t);
    meta[L.pos + t] = m.pos;
    meta[L.tok_seq + t] = m.seq;
    bool bad = false;
    meta[L.tokens + t] = resolve_token(tokens[t], tsrc, tsrc_len, vocab, &bad);
    if (bad) err |= 2;
    meta[L.slot + t] = m.slot;
  }
  for (int r = 0; r < R && r < cu_rows[S]; ++r) meta[L.rows + r] = row_token(cu_rows, cu_q, qlen, count, S, r);
  for (int i = 0; i < cu_tiles[S]; ++i) {  // phase 5
    const int s = upper_index(cu_tiles, S + 1, i);
    meta[L.tile_seq + i] = s;
    meta[L.tile_q0 + i] = (i - cu_tiles[s]) * qp;
  }
  cnt[kCntSeqs] = S;
  cnt[kCntTokens] = T;
  cnt[kCntRows] = R;
  cnt[kCntWidth] = W;
  cnt[kCntDecode] = cd;
  cnt[kCntTiles] = ct;
  cnt[kCntMaxCtx] = max_ctx;
  cnt[kCntMaxQlen] = max_q;
  return cnt[kCntError] = err;
}
