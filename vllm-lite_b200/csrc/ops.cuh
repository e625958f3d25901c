// Internal launchers shared by the C ABI and the forward orchestration.
#pragma once

#include "meta.cuh"

namespace vllt {

int reshape_and_cache(const void* k, const void* v, void* kc, void* vc, const int32_t* slots,
                      int num_tokens, int n_kv, int D, int bs, int num_blocks, int dtype,
                      cudaStream_t st);
int copy_blocks(void* kc, void* vc, const int32_t* pairs, int n_pairs, int n_layers,
                int num_blocks, int n_kv, int bs, int D, int dtype, cudaStream_t st);

int rmsnorm(const float* x, const int32_t* idx, const float* w, float* out, int rows_cap,
            const int32_t* rows_dev, int dim, float eps, cudaStream_t st);
int embed(const float* emb, const int32_t* tok, float* x, int T_cap, const int32_t* T_dev, int dim,
          int vocab, cudaStream_t st);
int embed_bf16(const void* emb, const int32_t* tok, float* x, int T_cap, const int32_t* T_dev, int dim,
               int vocab, cudaStream_t st);
int rmsnorm_bf16(float* x, const void* add, const int32_t* idx, const float* w, void* out, int rows_cap,
                 const int32_t* rows_dev, int dim, float eps, cudaStream_t st);
int argmax_rows(const float* logits, int rows_cap, const int32_t* rows_dev, int vocab, int ld, int offset,
                float* val, int32_t* idx, cudaStream_t st);
int rope(float* x, const int32_t* positions, const float* cos_t, const float* sin_t, int T,
         int heads, int D, int max_pos, cudaStream_t st);

int sample_greedy(const float* logits, int rows_cap, const int32_t* rows_dev, int vocab, int ld,
                  const uint8_t* eos_mask, int eos_id, const float* penalty, const uint32_t* seen,
                  int32_t* out, cudaStream_t st);
int spec_accept(const int32_t* cu_rows, const int32_t* drafts, const int32_t* draft_off,
                int num_seqs, const int32_t* picks, int32_t* n_accepted, cudaStream_t st);
int sample_top_p(const float* logits, int rows, int vocab, int ld, int logit_rows, const int32_t* row_index,
                 const uint8_t* eos_mask, int eos_id, const float* penalty, const uint32_t* seen,
                 const float* temperature, const int32_t* top_k, const float* top_p, const double* u,
                 int32_t* out, cudaStream_t st);

struct AttnCall {
  const void *q, *kc, *vc;
  void* out;
  const int32_t *tables, *cu_q, *ctx;
  int W, H, n_kv, D, bs, num_blocks, dtype;
  float scale;
  int P_cap;        // sequences the split-K partials are indexed by
  int T_rows;       // rows of q / out (the tensor-core prefill's Q map)
  float* ws;        // attention workspace: 256-byte flags header, then split partials
  int64_t ws_bytes;
  int* err;         // device error word (overrides the header's), may be NULL
};
int64_t attention_ws_bytes(int P_cap, int H, int D, int max_ctx);
// One attention pass. With item lists (forward): items_cap bounds the grid and
// the lists come from the meta builder. Without (standalone, item_seq == NULL):
// items are (sequence, tile) pairs derived from num_seqs and max_qlen.
int attention_pass(const AttnCall& c, const int32_t* item_seq, const int32_t* item_q0,
                   const int32_t* n_items, int items_cap, int num_seqs, int max_qlen,
                   bool single_query, int max_ctx, cudaStream_t st);
// Query positions per multi-token tile for this call's kernel (tensor-core
// prefill: 128 / n_rep; generic: 16 / n_rep).
int query_tile_positions(int dtype, int head_dim, int block_size, int n_rep);

}  // namespace vllt
