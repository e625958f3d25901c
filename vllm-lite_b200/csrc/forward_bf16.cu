// Forward pass of the bf16 (Llama-3-8B-shaped) model: the same pass as
// TinyLlama.forward (vllmlite/model.py:80-120) in bf16 with fp32 accumulation
// and an fp32 residual stream, optionally tensor-parallel.
//
// Per layer:
//   h  = rmsnorm(x)                          -> bf16           (fused residual add when tp > 1)
//   q,k,v = h . Wqkv^T  (tcgen05)            -> RoPE; q bf16, k/v into the bf16 paged cache
//   a  = paged attention(q)                  -> bf16  (TMA decode kernel / generic tiles)
//   x += a . Wo^T                            -> tp == 1: fp32 epilogue add
//                                               tp  > 1: bf16 partial, NCCL all-reduce, added by the next norm
//   h  = rmsnorm(x); act = silu(h.Wg^T) * (h.Wu^T) (one GEMM, interleaved columns) -> bf16
//   x += act . Wdown^T                       -> as o_proj
// then the final norm on the logit rows and lm_head (this rank's vocabulary rows).

#include <algorithm>

#include "gemm_bf16_tc.cuh"
#include "ops.cuh"

namespace vllt {

int tp_allreduce_bf16(void* buf, int64_t count, void* comm, cudaStream_t st);

namespace {

#define VLLT_TRY(expr)              \
  do {                              \
    const int _rc = (expr);         \
    if (_rc != VLLT_OK) return _rc; \
  } while (0)

struct Bf16Ws {
  float* x;              // [T][d] fp32 residual
  __nv_bfloat16* y;      // [T][d] bf16 partial (tp > 1)
  __nv_bfloat16* h;      // [T][d] normalized
  __nv_bfloat16* q;      // [T][H*D]
  __nv_bfloat16* attn;   // [T][H*D]
  __nv_bfloat16* act;    // [T][d_ff]
  __nv_bfloat16* rows_h; // [R][d]
  float* attn_ws;
  int64_t attn_ws_bytes, total_bytes;
  SplitKScratch sk;      // small-M projections: partial tiles + per-tile counters
};

Bf16Ws carve_bf16(const vllt_model_desc* m, const vllt_caps* c, char* base) {
  Bf16Ws w{};
  int64_t off = 0;
  auto take = [&](int64_t bytes) {
    char* p = base ? base + off : nullptr;
    off += align_up(bytes, 256);
    return p;
  };
  const int64_t T = c->max_tokens, R = c->max_rows, d = m->d_model;
  const int64_t qw = (int64_t)m->n_heads * m->head_dim;
  w.x = reinterpret_cast<float*>(take(T * d * 4));
  w.y = reinterpret_cast<__nv_bfloat16*>(take(m->tp_size > 1 ? T * d * 2 : 0));
  w.h = reinterpret_cast<__nv_bfloat16*>(take(T * d * 2));
  w.q = reinterpret_cast<__nv_bfloat16*>(take(T * qw * 2));
  w.attn = reinterpret_cast<__nv_bfloat16*>(take(T * qw * 2));
  w.act = reinterpret_cast<__nv_bfloat16*>(take(T * m->d_ff * 2));
  w.rows_h = reinterpret_cast<__nv_bfloat16*>(take(R * d * 2));
  w.attn_ws_bytes = attention_ws_bytes(c->max_seqs, m->n_heads, m->head_dim, m->max_seq_len);
  w.attn_ws = reinterpret_cast<float*>(take(w.attn_ws_bytes));
  w.sk = forward_splitk_scratch(nullptr);
  w.sk.part = reinterpret_cast<float*>(take(w.sk.part_bytes));
  w.sk.counters = reinterpret_cast<int*>(take((int64_t)w.sk.n_counters * 4));
  w.total_bytes = off;
  return w;
}

}  // namespace

int64_t forward_bf16_ws_bytes(const vllt_model_desc* m, const vllt_caps* c) {
  return carve_bf16(m, c, nullptr).total_bytes;
}

int forward_bf16(const vllt_model_desc* m, const int32_t* rec, const vllt_caps* caps, const vllt_step_bounds* b,
                 void* meta_v, void* ws, int64_t ws_bytes, float* logits, cudaStream_t st) {
  VLLT_REQUIRE(m->head_dim % 32 == 0 && m->d_model % 64 == 0 && m->d_ff % 64 == 0 &&
                   (m->n_heads * m->head_dim) % 64 == 0,
               "forward_bf16: head_dim must be a multiple of 32 and d_model, d_ff, n_heads*head_dim of 64");
  VLLT_REQUIRE(m->tp_size == 1 || m->tp_comm, "forward_bf16: tp_size > 1 needs tp_comm");
  const Bf16Ws w = carve_bf16(m, caps, reinterpret_cast<char*>(ws));
  VLLT_REQUIRE(ws_bytes >= w.total_bytes, "forward_bf16: workspace too small (%lld < %lld)", (long long)ws_bytes,
               (long long)w.total_bytes);
  const MetaLayout L = MetaLayout::make(caps->max_seqs, caps->max_tokens, caps->max_rows, caps->max_table_width);
  int32_t* meta = reinterpret_cast<int32_t*>(meta_v);
  int* err = meta + kCntError;
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
  const bool tp = m->tp_size > 1;

  VLLT_TRY(build_batch_meta(rec, L, m->block_size, m->num_blocks,
                            query_tile_positions(VLLT_BF16, D, m->block_size, n_rep), meta, st, m->table_pool,
                            m->table_pool_slots, m->token_source, m->token_source_len, m->embed_rows));
  VLLT_TRY(embed_bf16(m->tok_emb, meta + L.tokens, w.x, T_cap, T_dev, d, m->embed_rows, st));

  AttnCall ac{};
  ac.q = w.q;
  ac.out = w.attn;
  ac.tables = meta + L.tables;
  ac.W = L.W_cap;
  ac.cu_q = meta + L.cu_q;
  ac.ctx = meta + L.ctx;
  ac.H = H; ac.n_kv = KV; ac.D = D; ac.bs = m->block_size; ac.num_blocks = m->num_blocks;
  ac.dtype = VLLT_BF16;
  ac.scale = (float)(1.0 / sqrt((double)D));
  ac.P_cap = caps->max_seqs;
  ac.T_rows = caps->max_tokens;
  ac.ws = w.attn_ws;
  ac.ws_bytes = w.attn_ws_bytes;
  ac.err = err;

  const __nv_bfloat16* pending = nullptr;  // all-reduced partial still to join the residual (tp > 1)
  for (int l = 0; l < m->n_layers; ++l) {
    __nv_bfloat16* kc = reinterpret_cast<__nv_bfloat16*>(m->k_cache) + l * layer_elems;
    __nv_bfloat16* vc = reinterpret_cast<__nv_bfloat16*>(m->v_cache) + l * layer_elems;
    VLLT_TRY(rmsnorm_bf16(w.x, pending, nullptr, m->attn_norm[l], w.h, T_cap, T_dev, d, eps, st));
    pending = nullptr;
    EpiQKVBF16 eq{w.q, kc, vc, meta + L.pos, meta + L.slot, m->rope_cos, m->rope_sin,
                  H, KV, D, m->block_size, m->max_seq_len, (int64_t)m->num_blocks * m->block_size};
    VLLT_TRY(gemm_bf16_launch(w.h, T_cap, T_dev, m->wqkv[l], qkv_n, d, eq, err, st, &w.sk));
    ac.kc = kc;
    ac.vc = vc;
    VLLT_TRY(attention_pass(ac, meta + L.dec_seq, nullptr, meta + kCntDecode, dec_cap, 0, 0, true, max_ctx, st));
    VLLT_TRY(attention_pass(ac, meta + L.tile_seq, meta + L.tile_q0, meta + kCntTiles, tiles_cap, 0, 0, false,
                            max_ctx, st));
    if (tp) {
      VLLT_TRY(gemm_bf16_launch(w.attn, T_cap, T_dev, m->wo[l], d, H * D, EpiStoreBF16{w.y, d, d}, err, st, &w.sk));
      VLLT_TRY(tp_allreduce_bf16(w.y, (int64_t)T_cap * d, m->tp_comm, st));
      pending = w.y;
    } else {
      VLLT_TRY(gemm_bf16_launch(w.attn, T_cap, T_dev, m->wo[l], d, H * D, EpiResidualF32{w.x, d}, err, st, &w.sk));
    }
    VLLT_TRY(rmsnorm_bf16(w.x, pending, nullptr, m->ffn_norm[l], w.h, T_cap, T_dev, d, eps, st));
    pending = nullptr;
    VLLT_TRY(gemm_bf16_launch(w.h, T_cap, T_dev, m->w_gu[l], 2 * m->d_ff, d, EpiSwiGLUBF16{w.act, m->d_ff}, err,
                              st, &w.sk));
    if (tp) {
      VLLT_TRY(gemm_bf16_launch(w.act, T_cap, T_dev, m->w_down[l], d, m->d_ff, EpiStoreBF16{w.y, d, d}, err, st, &w.sk));
      VLLT_TRY(tp_allreduce_bf16(w.y, (int64_t)T_cap * d, m->tp_comm, st));
      pending = w.y;
    } else {
      VLLT_TRY(gemm_bf16_launch(w.act, T_cap, T_dev, m->w_down[l], d, m->d_ff, EpiResidualF32{w.x, d}, err, st, &w.sk));
    }
  }
  VLLT_TRY(rmsnorm_bf16(w.x, pending, meta + L.rows, m->final_norm, w.rows_h, R_cap, R_dev, d, eps, st));
  VLLT_TRY(gemm_bf16_launch(w.rows_h, R_cap, R_dev, m->lm_head, m->vocab, d,
                            EpiStoreF32{logits, m->vocab_padded, m->vocab}, err, st, &w.sk));
  return VLLT_OK;
}

}  // namespace vllt
