// The extern "C" surface declared in include/vllt.h, and the forward pass
// orchestration (TinyLlama.forward, vllmlite/model.py:80-120).

#include <stdarg.h>
#include <stdio.h>

#include <algorithm>
#include <atomic>

#include "gemm_f32.cuh"
#include "ops.cuh"

namespace vllt {

static thread_local char g_err[512] = "";
static std::atomic<int64_t> g_launches{0};

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
}
void clear_error() { g_err[0] = 0; }

int check_launch(const char* what) {
  g_launches.fetch_add(1, std::memory_order_relaxed);  // every launch site calls this once
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_error("%s: %s", what, cudaGetErrorString(e));
    return VLLT_ERR_CUDA;
  }
  return VLLT_OK;
}

int forward_bf16(const vllt_model_desc* m, const int32_t* rec, const vllt_caps* caps, const vllt_step_bounds* b,
                 void* meta_v, void* ws, int64_t ws_bytes, float* logits, cudaStream_t st);
int64_t forward_bf16_ws_bytes(const vllt_model_desc* m, const vllt_caps* caps);

namespace {

#define VLLT_TRY(expr)             \
  do {                             \
    const int _rc = (expr);        \
    if (_rc != VLLT_OK) return _rc; \
  } while (0)

bool caps_ok(const vllt_caps* c) {
  return c && c->max_seqs > 0 && c->max_tokens > 0 && c->max_rows > 0 && c->max_table_width > 0;
}

MetaLayout layout_of(const vllt_caps* c) {
  return MetaLayout::make(c->max_seqs, c->max_tokens, c->max_rows, c->max_table_width);
}

// Forward workspace carve-up (floats, 256-byte aligned pieces).
struct FwdWs {
  float *x, *h, *q, *attn, *act, *rows_h, *attn_ws;
  int64_t attn_ws_bytes, total_bytes;
  GemmScratch gemm;
};

FwdWs carve(const vllt_model_desc* m, const vllt_caps* c, char* base) {
  FwdWs w{};
  int64_t off = 0;
  auto take = [&](int64_t bytes) {
    char* p = base ? base + off : nullptr;
    off += align_up(bytes, 256);
    return reinterpret_cast<float*>(p);
  };
  const int64_t T = c->max_tokens, R = c->max_rows;
  const int64_t qw = (int64_t)m->n_heads * m->head_dim;
  w.x = take(T * m->d_model * 4);
  w.h = take(T * m->d_model * 4);
  w.q = take(T * qw * 4);
  w.attn = take(T * qw * 4);
  w.act = take(T * m->d_ff * 4);
  w.rows_h = take(R * m->d_model * 4);
  w.attn_ws_bytes = attention_ws_bytes(c->max_seqs, m->n_heads, m->head_dim, m->max_seq_len);
  w.attn_ws = take(w.attn_ws_bytes);
  const int n_max = std::max({(m->n_heads + 2 * m->n_kv_heads) * m->head_dim, 2 * m->d_ff, m->d_model,
                              m->vocab_padded});
  w.gemm.partial_floats = gemm_scratch_floats(n_max);
  w.gemm.n_counters = gemm_scratch_counters(n_max);
  w.gemm.partials = take(w.gemm.partial_floats * 4);
  w.gemm.counters = reinterpret_cast<int*>(take((int64_t)w.gemm.n_counters * 4));
  w.total_bytes = off;
  return w;
}

int check_desc(const vllt_model_desc* m) {
  VLLT_REQUIRE(m, "model desc is NULL");
  VLLT_REQUIRE(m->dtype == VLLT_F32 || m->dtype == VLLT_BF16, "vllt_forward: dtype must be F32 or BF16");
  VLLT_REQUIRE(m->tp_size >= 1 && (m->tp_size == 1 || m->dtype == VLLT_BF16),
               "vllt_forward: tensor parallelism is built for the bf16 model only");
  VLLT_REQUIRE(m->embed_rows >= (m->tp_size == 1 ? m->vocab : 1), "vllt_forward: embed_rows too small");
  VLLT_REQUIRE(!m->table_pool || m->table_pool_slots > 0, "vllt_forward: table_pool needs table_pool_slots > 0");
  VLLT_REQUIRE(!m->token_source || m->token_source_len > 0, "vllt_forward: token_source needs token_source_len > 0");
  VLLT_REQUIRE(m->n_layers > 0 && m->n_heads > 0 && m->n_kv_heads > 0 &&
                   m->n_heads % m->n_kv_heads == 0 && m->head_dim > 0 && m->d_model > 0 &&
                   m->d_ff > 0 && m->vocab > 0 && m->vocab_padded >= m->vocab &&
                   m->vocab_padded % 4 == 0 && m->block_size > 0 && m->num_blocks > 0 &&
                   m->max_seq_len > 0,
               "vllt_forward: bad model shape");
  // the attention kernels are built for these head sizes; checked before any
  // launch (each layer's QKV epilogue rotates and routes 4-column chunks, which
  // needs head_dim % 4 == 0, and runs before its attention)
  VLLT_REQUIRE(m->head_dim == 8 || m->head_dim == 16 || m->head_dim == 32 || m->head_dim == 48 ||
                   m->head_dim == 64 || m->head_dim == 128,
               "vllt_forward: head_dim %d not built (8, 16, 32, 48, 64, 128)", m->head_dim);
  VLLT_REQUIRE(m->d_model % 8 == 0 && m->d_ff % 4 == 0, "vllt_forward: d_model must be a multiple of 8 and d_ff of 4");
  VLLT_REQUIRE(m->tok_emb && m->final_norm && m->lm_head && m->rope_cos && m->rope_sin &&
                   m->attn_norm && m->wqkv && m->wo && m->ffn_norm && m->w_gu && m->w_down &&
                   m->k_cache && m->v_cache,
               "vllt_forward: null weight / cache pointer");
  for (int l = 0; l < m->n_layers; ++l)
    VLLT_REQUIRE(m->attn_norm[l] && m->wqkv[l] && m->wo[l] && m->ffn_norm[l] && m->w_gu[l] &&
                     m->w_down[l],
                 "vllt_forward: null weight in layer %d", l);
  return VLLT_OK;
}

int forward_impl(const vllt_model_desc* m, const int32_t* rec, const vllt_caps* caps,
                 const vllt_step_bounds* b, void* meta_v, void* ws, int64_t ws_bytes,
                 float* logits, cudaStream_t st) {
  VLLT_TRY(check_desc(m));
  VLLT_REQUIRE(caps_ok(caps) && b && rec && meta_v && ws && logits, "vllt_forward: bad arguments");
  if (m->dtype == VLLT_BF16) return forward_bf16(m, rec, caps, b, meta_v, ws, ws_bytes, logits, st);
  const FwdWs w = carve(m, caps, reinterpret_cast<char*>(ws));
  VLLT_REQUIRE(ws_bytes >= w.total_bytes, "vllt_forward: workspace too small (%lld < %lld)",
               (long long)ws_bytes, (long long)w.total_bytes);
  VLLT_REQUIRE(caps->max_table_width * m->block_size >= 1, "bad table width");
  const MetaLayout L = layout_of(caps);
  int32_t* meta = reinterpret_cast<int32_t*>(meta_v);
  const int n_rep = m->n_heads / m->n_kv_heads;
  const int T_cap = std::min(std::max(b->tokens, 0), caps->max_tokens);
  const int R_cap = std::min(std::max(b->rows, 0), caps->max_rows);
  const int dec_cap = std::min(std::max(b->decode_seqs, 0), caps->max_seqs);
  const int tiles_cap = std::min(std::max(b->tiles, 0), L.tiles_cap);
  const int max_ctx = std::min(std::max(b->max_ctx, 1), m->max_seq_len);
  const int32_t* T_dev = meta + kCntTokens;
  const int32_t* R_dev = meta + kCntRows;
  const int d = m->d_model, H = m->n_heads, KV = m->n_kv_heads, D = m->head_dim;
  const int qkv_n = (H + 2 * KV) * D;
  const int64_t layer_elems = (int64_t)m->num_blocks * KV * m->block_size * D;
  const float eps = m->rms_eps;

  VLLT_TRY(build_batch_meta(rec, L, m->block_size, m->num_blocks,
                            query_tile_positions(VLLT_F32, D, m->block_size, n_rep), meta, st, m->table_pool,
                            m->table_pool_slots, m->token_source, m->token_source_len, m->vocab));
  VLLT_TRY(embed(reinterpret_cast<const float*>(m->tok_emb), meta + L.tokens, w.x, T_cap, T_dev, d, m->vocab, st));

  AttnCall ac{};
  ac.q = w.q;
  ac.out = w.attn;
  ac.tables = meta + L.tables;
  ac.W = L.W_cap;
  ac.cu_q = meta + L.cu_q;
  ac.ctx = meta + L.ctx;
  ac.H = H; ac.n_kv = KV; ac.D = D; ac.bs = m->block_size; ac.num_blocks = m->num_blocks;
  ac.dtype = VLLT_F32;
  ac.scale = (float)(1.0 / sqrt((double)D));  // float64 then rounded, as model.py:58
  ac.P_cap = caps->max_seqs;
  ac.T_rows = caps->max_tokens;
  ac.ws = w.attn_ws;
  ac.ws_bytes = w.attn_ws_bytes;
  ac.err = meta + kCntError;  // bounded-wait timeouts surface in the step's error counter

  for (int l = 0; l < m->n_layers; ++l) {
    float* kc = reinterpret_cast<float*>(m->k_cache) + l * layer_elems;
    float* vc = reinterpret_cast<float*>(m->v_cache) + l * layer_elems;
    // h = rms_norm(x) ; q,k,v = h @ [wq|wk|wv] ; rope ; k,v -> cache
    VLLT_TRY(rmsnorm(w.x, nullptr, m->attn_norm[l], w.h, T_cap, T_dev, d, eps, st));
    EpiQKV eq{w.q, kc, vc, meta + L.pos, meta + L.slot, m->rope_cos, m->rope_sin,
              H, KV, D, m->block_size, m->max_seq_len, (int64_t)m->num_blocks * m->block_size};
    VLLT_TRY(sgemm_launch(w.h, d, reinterpret_cast<const float*>(m->wqkv[l]), qkv_n, T_cap, T_dev, qkv_n, d, eq, st,
                          &w.gemm));
    // attention: single-query sequences, then multi-token tiles
    ac.kc = kc;
    ac.vc = vc;
    VLLT_TRY(attention_pass(ac, meta + L.dec_seq, nullptr, meta + kCntDecode, dec_cap, 0, 0, true,
                            max_ctx, st));
    VLLT_TRY(attention_pass(ac, meta + L.tile_seq, meta + L.tile_q0, meta + kCntTiles, tiles_cap,
                            0, 0, false, max_ctx, st));
    // x += attn @ wo
    VLLT_TRY(sgemm_launch(w.attn, H * D, reinterpret_cast<const float*>(m->wo[l]), d, T_cap, T_dev, d, H * D,
                          EpiResidual{w.x, d}, st, &w.gemm));
    // x += (silu(h @ w_gate) * (h @ w_up)) @ w_down
    VLLT_TRY(rmsnorm(w.x, nullptr, m->ffn_norm[l], w.h, T_cap, T_dev, d, eps, st));
    VLLT_TRY(sgemm_launch(w.h, d, reinterpret_cast<const float*>(m->w_gu[l]), 2 * m->d_ff, T_cap, T_dev, 2 * m->d_ff, d,
                          EpiSwiGLU{w.act, m->d_ff}, st, &w.gemm));
    VLLT_TRY(sgemm_launch(w.act, m->d_ff, reinterpret_cast<const float*>(m->w_down[l]), d, T_cap, T_dev, d, m->d_ff,
                          EpiResidual{w.x, d}, st, &w.gemm));
  }
  // logits only for the wanted rows (model.py:119-120)
  VLLT_TRY(rmsnorm(w.x, meta + L.rows, m->final_norm, w.rows_h, R_cap, R_dev, d, eps, st));
  VLLT_TRY(sgemm_launch(w.rows_h, d, reinterpret_cast<const float*>(m->lm_head), m->vocab_padded, R_cap, R_dev,
                        m->vocab_padded, d,
                        EpiStore{logits, m->vocab_padded, m->vocab_padded}, st, &w.gemm));
  return VLLT_OK;
}

}  // namespace
}  // namespace vllt

using namespace vllt;

extern "C" {

const char* vllt_last_error(void) { return g_err; }
int vllt_version(void) { return 100; }
int64_t vllt_kernel_launches(void) { return g_launches.load(); }

int vllt_reshape_and_cache(const void* k, const void* v, void* k_cache, void* v_cache,
                           const int32_t* slot_mapping, int32_t num_tokens, int32_t n_kv,
                           int32_t head_dim, int32_t block_size, int32_t num_blocks,
                           int32_t dtype, void* stream) {
  clear_error();
  VLLT_REQUIRE(num_tokens >= 0 && n_kv > 0 && head_dim > 0 && block_size > 0 && num_blocks > 0,
               "reshape_and_cache: bad sizes");
  VLLT_REQUIRE(dtype == VLLT_F32 || dtype == VLLT_BF16, "reshape_and_cache: bad dtype");
  if (num_tokens == 0) return VLLT_OK;
  VLLT_REQUIRE(k && v && k_cache && v_cache && slot_mapping, "reshape_and_cache: null pointer");
  return reshape_and_cache(k, v, k_cache, v_cache, slot_mapping, num_tokens, n_kv, head_dim,
                           block_size, num_blocks, dtype, as_stream(stream));
}

int vllt_copy_blocks(void* k_cache, void* v_cache, const int32_t* pairs, int32_t n_pairs,
                     int32_t n_layers, int32_t num_blocks, int32_t n_kv, int32_t block_size,
                     int32_t head_dim, int32_t dtype, void* stream) {
  clear_error();
  VLLT_REQUIRE(n_pairs >= 0 && n_layers > 0 && num_blocks > 0 && n_kv > 0 && block_size > 0 &&
                   head_dim > 0,
               "copy_blocks: bad sizes");
  VLLT_REQUIRE(dtype == VLLT_F32 || dtype == VLLT_BF16, "copy_blocks: bad dtype");
  if (n_pairs == 0) return VLLT_OK;
  VLLT_REQUIRE(k_cache && v_cache && pairs, "copy_blocks: null pointer");
  return copy_blocks(k_cache, v_cache, pairs, n_pairs, n_layers, num_blocks, n_kv, block_size,
                     head_dim, dtype, as_stream(stream));
}

int64_t vllt_meta_bytes(const vllt_caps* caps) {
  if (!caps_ok(caps)) return -1;
  return layout_of(caps).words * 4;
}

int vllt_build_batch_meta(const int32_t* step_record, const vllt_caps* caps, int32_t block_size,
                          int32_t num_blocks, int32_t n_rep, void* meta, void* stream) {
  clear_error();
  VLLT_REQUIRE(caps_ok(caps), "build_batch_meta: bad capacities");
  VLLT_REQUIRE(n_rep > 0, "build_batch_meta: bad n_rep");
  return build_batch_meta(step_record, layout_of(caps), block_size, num_blocks, tile_positions(n_rep),
                          reinterpret_cast<int32_t*>(meta), as_stream(stream));
}

int vllt_build_batch_meta_pooled(const int32_t* step_record, const vllt_caps* caps, int32_t block_size,
                                 int32_t num_blocks, int32_t n_rep, int32_t* table_pool, int32_t pool_slots,
                                 void* meta, void* stream) {
  clear_error();
  VLLT_REQUIRE(caps_ok(caps), "build_batch_meta: bad capacities");
  VLLT_REQUIRE(n_rep > 0, "build_batch_meta: bad n_rep");
  VLLT_REQUIRE(table_pool && pool_slots > 0, "build_batch_meta: the pooled record needs a table pool");
  return build_batch_meta(step_record, layout_of(caps), block_size, num_blocks, tile_positions(n_rep),
                          reinterpret_cast<int32_t*>(meta), as_stream(stream), table_pool, pool_slots);
}

int32_t* vllt_meta_field(void* meta, const vllt_caps* caps, int32_t which) {
  if (!meta || !caps_ok(caps)) return nullptr;
  const MetaLayout L = layout_of(caps);
  int32_t* m = reinterpret_cast<int32_t*>(meta);
  switch (which) {
    case 0: return m;
    case 1: return m + L.cu_q;
    case 2: return m + L.cu_rows;
    case 3: return m + L.ctx;
    case 4: return m + L.pos;
    case 5: return m + L.slot;
    case 6: return m + L.rows;
    case 7: return m + L.tables;
    case 8: return m + L.tokens;
    default: return nullptr;
  }
}

int64_t vllt_attention_workspace_bytes(int32_t num_seqs, int32_t n_heads, int32_t head_dim,
                                       int32_t max_ctx) {
  return attention_ws_bytes(num_seqs, n_heads, head_dim, max_ctx);
}

int vllt_paged_attention_varlen(const void* q, const void* k_cache, const void* v_cache,
                                const int32_t* block_tables, int32_t table_width,
                                const int32_t* cu_seqlens_q, const int32_t* ctx_lens,
                                int32_t num_seqs, int32_t num_tokens, int32_t max_qlen,
                                int32_t max_ctx, int32_t n_heads, int32_t n_kv,
                                int32_t head_dim, int32_t block_size, int32_t num_blocks,
                                float scale, int32_t dtype, void* out, void* workspace,
                                int64_t workspace_bytes, void* stream) {
  clear_error();
  VLLT_REQUIRE(num_seqs >= 0 && num_tokens >= 0 && max_qlen >= 0 && max_ctx >= 0 && n_heads > 0 &&
                   n_kv > 0 && n_heads % n_kv == 0 && head_dim > 0 && block_size > 0 &&
                   num_blocks > 0 && table_width > 0,
               "paged_attention: bad sizes");
  VLLT_REQUIRE(dtype == VLLT_F32 || dtype == VLLT_BF16, "paged_attention: bad dtype");
  if (num_seqs == 0 || num_tokens == 0) return VLLT_OK;
  VLLT_REQUIRE(q && k_cache && v_cache && block_tables && cu_seqlens_q && ctx_lens && out,
               "paged_attention: null pointer");
  AttnCall c{};
  c.q = q; c.kc = k_cache; c.vc = v_cache; c.out = out;
  c.tables = block_tables; c.W = table_width; c.cu_q = cu_seqlens_q; c.ctx = ctx_lens;
  c.H = n_heads; c.n_kv = n_kv; c.D = head_dim; c.bs = block_size; c.num_blocks = num_blocks;
  c.dtype = dtype; c.scale = scale; c.P_cap = num_seqs;
  c.ws = reinterpret_cast<float*>(workspace);
  c.ws_bytes = workspace ? workspace_bytes : 0;
  c.err = nullptr;  // the workspace header carries the error word
  c.T_rows = num_tokens;
  // a pure decode batch (max_qlen <= 1) is one single-query item per sequence (split-K allowed)
  return attention_pass(c, nullptr, nullptr, nullptr, 0, num_seqs, max_qlen, max_qlen <= 1, max_ctx,
                        as_stream(stream));
}

int vllt_rmsnorm(const float* x, const int32_t* idx, const float* w, float* out, int32_t rows,
                 int32_t dim, float eps, void* stream) {
  clear_error();
  VLLT_REQUIRE(rows >= 0 && dim > 0, "rmsnorm: bad sizes");
  if (rows == 0) return VLLT_OK;
  VLLT_REQUIRE(x && w && out, "rmsnorm: null pointer");
  return rmsnorm(x, idx, w, out, rows, nullptr, dim, eps, as_stream(stream));
}

int vllt_rope(float* x, const int32_t* positions, const float* cos_t, const float* sin_t,
              int32_t num_tokens, int32_t heads, int32_t head_dim, int32_t max_pos, void* stream) {
  clear_error();
  VLLT_REQUIRE(num_tokens >= 0 && heads > 0 && head_dim > 0 && max_pos > 0, "rope: bad sizes");
  if (num_tokens == 0) return VLLT_OK;
  VLLT_REQUIRE(x && positions && cos_t && sin_t, "rope: null pointer");
  return rope(x, positions, cos_t, sin_t, num_tokens, heads, head_dim, max_pos, as_stream(stream));
}

int vllt_sgemm(const float* A, const float* B, float* C, int32_t M, int32_t N, int32_t K,
               void* stream) {
  clear_error();
  VLLT_REQUIRE(M >= 0 && N > 0 && K > 0, "sgemm: bad sizes");
  if (M == 0) return VLLT_OK;
  VLLT_REQUIRE(A && B && C, "sgemm: null pointer");
  return sgemm_launch(A, K, B, N, M, nullptr, N, K, EpiStore{C, N, N}, as_stream(stream));
}

int vllt_sample_greedy(const float* logits, int32_t rows, int32_t vocab, int32_t ld,
                       const uint8_t* eos_mask, int32_t eos_id, const float* penalty,
                       const uint32_t* seen_bits, int32_t* out_tokens, void* stream) {
  clear_error();
  VLLT_REQUIRE(rows >= 0 && vocab > 0 && ld >= vocab, "sample_greedy: bad sizes");
  if (rows == 0) return VLLT_OK;
  VLLT_REQUIRE(logits && out_tokens, "sample_greedy: null pointer");
  return sample_greedy(logits, rows, nullptr, vocab, ld, eos_mask, eos_id, penalty, seen_bits,
                       out_tokens, as_stream(stream));
}

int vllt_sample_top_p(const float* logits, int32_t rows, int32_t vocab, int32_t ld, int32_t logit_rows,
                      const int32_t* row_index, const uint8_t* eos_mask, int32_t eos_id, const float* penalty,
                      const uint32_t* seen_bits, const float* temperature, const int32_t* top_k,
                      const float* top_p, const double* u, int32_t* out_tokens, void* stream) {
  clear_error();
  VLLT_REQUIRE(rows >= 0 && vocab > 0 && ld >= vocab && logit_rows >= 0, "sample_top_p: bad sizes");
  if (rows == 0) return VLLT_OK;
  VLLT_REQUIRE(logit_rows > 0 && (row_index || rows <= logit_rows), "sample_top_p: more rows than logit_rows");
  VLLT_REQUIRE(logits && temperature && u && out_tokens, "sample_top_p: null pointer");
  return sample_top_p(logits, rows, vocab, ld, logit_rows, row_index, eos_mask, eos_id, penalty, seen_bits,
                      temperature, top_k, top_p, u, out_tokens, as_stream(stream));
}

int vllt_spec_verify(const float* logits, int32_t ld, int32_t vocab, const int32_t* cu_rows,
                     int32_t total_rows, const int32_t* drafts, const int32_t* draft_offsets,
                     int32_t num_seqs, int32_t* out_tokens, int32_t* n_accepted, void* stream) {
  clear_error();
  VLLT_REQUIRE(num_seqs >= 0 && total_rows >= num_seqs && vocab > 0 && ld >= vocab,
               "spec_verify: bad sizes");
  if (num_seqs == 0) return VLLT_OK;
  VLLT_REQUIRE(logits && cu_rows && draft_offsets && out_tokens && n_accepted,
               "spec_verify: null pointer");
  cudaStream_t st = as_stream(stream);
  const int rc = sample_greedy(logits, total_rows, nullptr, vocab, ld, nullptr, 0, nullptr, nullptr,
                               out_tokens, st);
  if (rc != VLLT_OK) return rc;
  return spec_accept(cu_rows, drafts, draft_offsets, num_seqs, out_tokens, n_accepted, st);
}

int vllt_argmax_rows(const float* logits, int32_t rows, int32_t vocab, int32_t ld, int32_t vocab_offset,
                     float* out_val, int32_t* out_idx, void* stream) {
  clear_error();
  VLLT_REQUIRE(rows >= 0 && vocab > 0 && ld >= vocab, "argmax_rows: bad sizes");
  if (rows == 0) return VLLT_OK;
  VLLT_REQUIRE(logits && out_val && out_idx, "argmax_rows: null pointer");
  return argmax_rows(logits, rows, nullptr, vocab, ld, vocab_offset, out_val, out_idx, as_stream(stream));
}

int vllt_spec_accept(const int32_t* cu_rows, const int32_t* drafts, const int32_t* draft_offsets,
                     int32_t num_seqs, const int32_t* picks, int32_t* n_accepted, void* stream) {
  clear_error();
  VLLT_REQUIRE(num_seqs >= 0, "spec_accept: bad sizes");
  if (num_seqs == 0) return VLLT_OK;
  VLLT_REQUIRE(cu_rows && drafts && draft_offsets && picks && n_accepted, "spec_accept: null pointer");
  return spec_accept(cu_rows, drafts, draft_offsets, num_seqs, picks, n_accepted, as_stream(stream));
}

int32_t vllt_query_tile_positions(const vllt_model_desc* m) {
  if (!m || m->n_kv_heads <= 0 || m->n_heads % m->n_kv_heads) return -1;
  return query_tile_positions(m->dtype, m->head_dim, m->block_size, m->n_heads / m->n_kv_heads);
}

int64_t vllt_forward_workspace_bytes(const vllt_model_desc* m, const vllt_caps* caps) {
  if (!m || !caps_ok(caps)) return -1;
  if (m->dtype == VLLT_BF16) return forward_bf16_ws_bytes(m, caps);
  return carve(m, caps, nullptr).total_bytes;
}

int vllt_forward(const vllt_model_desc* m, const int32_t* step_record, const vllt_caps* caps,
                 const vllt_step_bounds* bounds, void* meta, void* workspace,
                 int64_t workspace_bytes, float* logits, void* stream) {
  clear_error();
  return forward_impl(m, step_record, caps, bounds, meta, workspace, workspace_bytes, logits,
                      as_stream(stream));
}

}  // extern "C"
