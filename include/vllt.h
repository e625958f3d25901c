/*
 * vllt.h -- C ABI of the B200 (sm_100a) forward hot path for vllm-lite.
 *
 * Every entry point:
 *   - takes plain device pointers, sizes and a CUDA stream passed as `void*`
 *     (a cudaStream_t; NULL = the legacy default stream);
 *   - is stream-ordered and asynchronous: it validates its arguments on the
 *     host, enqueues kernels and returns;
 *   - returns an int status (VLLT_OK = 0). On failure the thread-local
 *     message is available from vllt_last_error().
 *   - allocates no device memory: callers pass every buffer, including
 *     workspaces sized by the *_bytes() helpers.
 *
 * KV cache layout (one layer): [num_blocks][n_kv_heads][block_size][head_dim],
 * i.e. one block of one KV head is a contiguous block_size x head_dim tile.
 * A "slot" is the reference's flat cache index block_id * block_size + offset
 * (vllmlite/attention.py:40-44, vllmlite/block.py:154-156). With block_size 1
 * the layout equals the reference's per-layer cache [slots][n_kv][head_dim]
 * (vllmlite/runner.py:41-44).
 *
 * Weights use the reference's row-major [in][out] orientation
 * (vllmlite/model.py:34-43); the fused matrices are documented at
 * vllt_model_desc.
 */
#ifndef VLLT_H_
#define VLLT_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  VLLT_OK = 0,
  VLLT_ERR_ARG = 1,         /* bad pointer / size / unsupported shape */
  VLLT_ERR_CUDA = 2,        /* a CUDA call or launch failed */
  VLLT_ERR_TIMEOUT = 3,     /* a bounded device-side wait expired */
  VLLT_ERR_UNSUPPORTED = 4, /* valid request this build does not implement */
  VLLT_ERR_DATA = 5         /* device-side validation flagged bad metadata */
};

enum { VLLT_F32 = 0, VLLT_BF16 = 1 };

/* Last error message of the calling thread ("" when none). */
const char* vllt_last_error(void);
/* Library version, major*10000 + minor*100 + patch. */
int vllt_version(void);
/* Kernels this library has launched in the process so far (all threads). */
int64_t vllt_kernel_launches(void);

/* ------------------------------------------------------------------------ */
/* KV cache                                                                 */
/* ------------------------------------------------------------------------ */

/* Scatter new K/V rows into the paged cache through a slot mapping.
 * Replaces write_kv (vllmlite/attention.py:47-49):
 *   cache[slot_mapping[t]] = k[t], v[t]   for t < num_tokens.
 * k, v: [num_tokens][n_kv][head_dim] of `dtype`. Slots outside
 * [0, num_blocks*block_size) are skipped by the kernel (never written). */
int vllt_reshape_and_cache(const void* k, const void* v, void* k_cache, void* v_cache,
                           const int32_t* slot_mapping, int32_t num_tokens, int32_t n_kv,
                           int32_t head_dim, int32_t block_size, int32_t num_blocks,
                           int32_t dtype, void* stream);

/* Copy whole blocks src -> dst in every layer, K and V, before any KV write of
 * the step. Replaces NumpyRunner._do_cow (vllmlite/runner.py:54-60).
 * pairs: device int32 [n_pairs][2] = (src_block, dst_block).
 * k_cache/v_cache: base of [n_layers][num_blocks][n_kv][block_size][head_dim]. */
int vllt_copy_blocks(void* k_cache, void* v_cache, const int32_t* pairs, int32_t n_pairs,
                     int32_t n_layers, int32_t num_blocks, int32_t n_kv, int32_t block_size,
                     int32_t head_dim, int32_t dtype, void* stream);

/* ------------------------------------------------------------------------ */
/* Batch flatten (ModelRunner.execute, vllmlite/runner.py:66-90)            */
/* ------------------------------------------------------------------------ */

/* A packed step record (device int32), written by the host once per pass:
 *   [0]=num_seqs S  [1]=num_tokens T  [2]=num_rows R  [3]=table width W
 *   seq_start[S]   position of the first token pushed this pass (num_computed)
 *   seq_qlen[S]    tokens pushed this pass (ScheduledSeq.num_tokens)
 *   seq_count[S]   logit rows wanted: min(1 + num_drafts, qlen) (runner.py:88)
 *   token_ids[T]   the pushed tokens, sequence after sequence
 *   block_tables[S][W]  physical block ids (BlockTable.block_ids), padded
 * Its length is 4 + 3*S + T + S*W int32 words.
 *
 * A token id t < 0 stands for entry -t - 1 of the forward's token source
 * (vllt_model_desc.token_source): a token the previous pass picked on the
 * device and the host has not read yet. The metadata builder resolves it; an
 * id outside [0, embed_rows) after that, or a reference outside the source,
 * embeds token 0 and sets error bit 1. Without a token source (and in the
 * vllt_build_batch_meta* entries) a negative id is such an error.
 *
 * The pooled record leaves the block tables on the device. A persistent pool
 * [pool_slots][max_table_width] int32 (allocated by the caller, contents
 * initially irrelevant) holds one table per live sequence; each pass carries
 * only what changed since the last (the blocks BlockManager.append_slots
 * appended or replaced by copy-on-write, vllmlite/block_manager.py:65-93, or a
 * whole table when a sequence first takes a slot):
 *   [0]=S [1]=T [2]=R [3]=W [4]=U (updates)
 *   seq_start[S], seq_qlen[S], seq_count[S], token_ids[T]   as above
 *   table_slot[S]  the pool row of each sequence
 *   updates[U][3]  (pool row, table index, block id), applied before the
 *                  tables are read; U <= max_seqs * max_table_width
 * Its length is 5 + 4*S + T + 3*U words. A pass reads entries
 * [0, ceil(ctx/block_size)) of each sequence's row; the rest of a row is
 * never read. */

/* Capacities of the buffers one runner allocates once. */
typedef struct vllt_caps {
  int32_t max_seqs;        /* S <= max_seqs */
  int32_t max_tokens;      /* T <= max_tokens */
  int32_t max_rows;        /* R <= max_rows */
  int32_t max_table_width; /* W <= max_table_width (= ceil(max_seq_len / block_size)) */
} vllt_caps;

/* Bytes of the opaque batch-metadata buffer for the given capacities. */
int64_t vllt_meta_bytes(const vllt_caps* caps);

/* Build, on the device, everything the forward pass indexes by:
 * cu_seqlens, per-token positions / flat slots / sequence ids, logit-row
 * token indices, context lengths and the attention work lists.
 * Positions follow runner.py:75 (start..start+qlen-1), slots follow
 * gather_slots (attention.py:40-44), rows follow runner.py:86-90.
 * A block id outside [0, num_blocks) or a context beyond the table marks the
 * slot -1 and sets the device error flag (counter 7, below). */
int vllt_build_batch_meta(const int32_t* step_record, const vllt_caps* caps, int32_t block_size,
                          int32_t num_blocks, int32_t n_rep, void* meta, void* stream);

/* The same from a pooled record: applies its updates to table_pool
 * ([pool_slots][caps->max_table_width] int32, device) and reads each
 * sequence's table from its pool row. An update or a table slot outside the
 * pool sets error bit 1. No reference counterpart beyond what
 * vllt_build_batch_meta replaces: it moves the block-table upload of
 * runner.py:66-90 from S*W words per pass to the changed entries. */
int vllt_build_batch_meta_pooled(const int32_t* step_record, const vllt_caps* caps, int32_t block_size,
                                 int32_t num_blocks, int32_t n_rep, int32_t* table_pool, int32_t pool_slots,
                                 void* meta, void* stream);

/* Device pointers into the meta buffer (for callers that launch their own
 * kernels on it): which = 0 counters[16], 1 cu_seqlens_q[S+1], 2 cu_rows[S+1],
 * 3 ctx_lens[S], 4 positions[T], 5 slot_mapping[T], 6 logit-row token
 * indices[R], 7 block tables [max_seqs][max_table_width], 8 token ids[T] (as
 * resolved: references to the token source replaced by the tokens). NULL if
 * unknown. */
int32_t* vllt_meta_field(void* meta, const vllt_caps* caps, int32_t which);

/* Counters: 0 S, 1 T, 2 R, 3 W, 4 single-query sequences, 5 query tiles,
 * 6 max context, 7 error flags (bit 0 capacity, bit 1 block table / range). */

/* ------------------------------------------------------------------------ */
/* Attention                                                                */
/* ------------------------------------------------------------------------ */

/* Workspace bytes for vllt_paged_attention_varlen: a 256-byte header whose
 * first int32 receives device error flags (bit 2: a bounded wait on a TMA
 * copy expired; zero it before a call to observe that call), then split-K
 * partials for long single-query contexts (indexed by sequence). */
int64_t vllt_attention_workspace_bytes(int32_t num_seqs, int32_t n_heads, int32_t head_dim,
                                       int32_t max_ctx);

/* Varlen causal paged attention over a ragged batch (decode, chunked
 * prefill and speculative-verify rows mixed). Replaces paged_attention
 * (vllmlite/attention.py:59-98) applied per sequence by the loop at
 * vllmlite/model.py:105-112.
 *   q    [num_tokens][n_heads][head_dim]   (dtype)
 *   out  [num_tokens][n_heads][head_dim]   (dtype)
 *   caches: one layer, layout in the file header (dtype)
 *   block_tables [num_seqs][table_width], cu_seqlens_q [num_seqs+1],
 *   ctx_lens [num_seqs] (tokens in the cache including this pass's).
 * Query j of sequence s sits at position ctx_lens[s] - qlen_s + j and sees
 * keys 0..that position; head h reads KV head h / (n_heads / n_kv).
 * max_qlen and max_ctx bound the work launched. With a NULL workspace the
 * generic kernel walks each context in one CTA (no split-K, no TMA path);
 * single-query bf16 work with head_dim 128 and block_size 16 takes the TMA
 * decode kernel when a workspace is given. */
int vllt_paged_attention_varlen(const void* q, const void* k_cache, const void* v_cache,
                                const int32_t* block_tables, int32_t table_width,
                                const int32_t* cu_seqlens_q, const int32_t* ctx_lens,
                                int32_t num_seqs, int32_t num_tokens, int32_t max_qlen,
                                int32_t max_ctx, int32_t n_heads, int32_t n_kv,
                                int32_t head_dim, int32_t block_size, int32_t num_blocks,
                                float scale, int32_t dtype, void* out, void* workspace,
                                int64_t workspace_bytes, void* stream);

/* The same attention, for callers that cannot allocate device memory: it
 * takes no workspace and keeps its split-K scratch and error word in a static
 * device array inside this library. No counterpart in the reference (which has
 * no device code); it exists for integrations that run under a device-memory
 * budget owned by someone else, that must not call cudaMalloc on their hot path
 * (cudaMalloc can synchronize the device), or whose interface hands them only
 * input and output buffers.
 *   - Scratch: 16 MiB per device, held by every GPU that loads the library
 *     until the process exits. A batch needing more (vllt_attention_workspace_bytes
 *     > 16 MiB, e.g. ~250 single-query sequences x 32 heads at 4096 context) is
 *     rejected with VLLT_ERR_ARG.
 *   - The first call on a device looks up the array's device address
 *     (cudaGetSymbolAddress, with that device current); make that first call
 *     before any stream capture. The address is kept for the process: after
 *     cudaDeviceReset on a device, do not call this entry point on it again.
 *   - Every call shares the one array and it keeps the last call's contents;
 *     the error word is cleared at the start of each call. Calls that overlap
 *     on the GPU (other streams, other threads) race on it: serialize them.
 *   - device_flags (optional device int32) receives the call's error flags
 *     (bit 2: a bounded wait on a TMA copy expired); an empty batch writes 0.
 * Allocates nothing: no cudaMalloc / cudaFree, no allocating library call. */
int vllt_paged_attention_varlen_noalloc(const void* q, const void* k_cache, const void* v_cache,
                                        const int32_t* block_tables, int32_t table_width,
                                        const int32_t* cu_seqlens_q, const int32_t* ctx_lens,
                                        int32_t num_seqs, int32_t num_tokens, int32_t max_qlen,
                                        int32_t max_ctx, int32_t n_heads, int32_t n_kv,
                                        int32_t head_dim, int32_t block_size, int32_t num_blocks,
                                        float scale, int32_t dtype, void* out,
                                        int32_t* device_flags, void* stream);

/* Test injection for the decode kernel's bounded waits (no reference
 * counterpart). The next TMA-decode launch made by this thread (through
 * vllt_paged_attention_varlen or vllt_forward) arms the mbarrier of the stage
 * that would hold table index `table_index` for its bytes but issues no copy
 * into it, and limits every wait of that launch to wait_ns (<= 1 s): each
 * CTA reading that index sees its wait expire, sets error bit 2 in the
 * workspace flags, waits for its other copies in flight and returns; the
 * context stays usable. One-shot: later launches wait normally; a launch
 * captured into a CUDA graph neither takes nor consumes the injection. */
int vllt_test_decode_stall(int32_t table_index, int64_t wait_ns);

/* ------------------------------------------------------------------------ */
/* Layer pieces                                                             */
/* ------------------------------------------------------------------------ */

/* out[r] = x[idx[r]] / sqrt(mean(x[idx[r]]^2) + eps) * w; idx may be NULL
 * (identity). fp32. Replaces rms_norm (vllmlite/model.py:17-19). */
int vllt_rmsnorm(const float* x, const int32_t* idx, const float* w, float* out,
                 int32_t rows, int32_t dim, float eps, void* stream);

/* Interleaved-pair rotary embedding in place on x [T][heads][head_dim] (fp32)
 * with tables cos/sin [max_pos][head_dim/2]. Replaces apply_rope
 * (vllmlite/attention.py:28-37). */
int vllt_rope(float* x, const int32_t* positions, const float* cos_t, const float* sin_t,
              int32_t num_tokens, int32_t heads, int32_t head_dim, int32_t max_pos,
              void* stream);

/* C[M][N] = A[M][K] @ B[K][N] (fp32, row-major, CUDA-core FFMA, no TF32).
 * The parity-mode GEMM behind every projection of vllmlite/model.py:98-120. */
int vllt_sgemm(const float* A, const float* B, float* C, int32_t M, int32_t N, int32_t K,
               void* stream);

/* C[M][N] = A[M][K] . W[N][K]^T on the tcgen05 tensor cores: bf16 A and W (both
 * K-major, i.e. W is stored [out][in]), fp32 accumulate in tensor memory, fp32 C.
 * K must be a multiple of 64; device_flags (device int32) receives bit 2 if a
 * bounded wait expired. The bf16 projections of the Llama-3-8B-shaped model
 * (the bf16 counterpart of vllmlite/model.py:98-120) run on this kernel. */
int vllt_gemm_bf16(const void* A, const void* W, float* C, int32_t M, int32_t N, int32_t K,
                   int32_t* device_flags, void* stream);

/* The same GEMM in the forms the forward pass uses for few token rows:
 *   splits >= 2: K cut into `splits` slices (splits <= K/64), one CTA per
 *     (tile, slice); the last slice of each tile to finish sums the fp32
 *     partials in slice order (deterministic) and writes C;
 *   splits <= 0: the forward's own choice for (M, N, K). For M <= 256 (N a
 *     multiple of 32) the weights go on the MMA's M side (128 features x all
 *     tokens per CTA) and either the CTAs of a thread-block cluster split K
 *     for one feature tile and sum their accumulators through distributed
 *     shared memory (few tiles), or the (feature tile, k-block) iterations are
 *     divided evenly over one CTA per SM and split tiles summed in CTA order
 *     by a second kernel (stream-K); otherwise split-K as
 *     vllt_gemm_bf16_auto_splits says, else the persistent kernel;
 *   splits == 1: the persistent kernel (as vllt_gemm_bf16).
 * `workspace` (device, at least vllt_gemm_bf16_splitk_workspace_bytes(M, N, K,
 * splits) bytes) must be zero before its first use and is left reusable.
 * vllt_gemm_bf16_auto_splits returns -S for the cluster form (S CTAs per
 * feature tile), 0 for the stream-K form, else the split count. No reference counterpart (vllm-lite multiplies with NumPy);
 * these expose the forward's small-M paths to tests and callers. */
int64_t vllt_gemm_bf16_splitk_workspace_bytes(int32_t M, int32_t N, int32_t K, int32_t splits);
int32_t vllt_gemm_bf16_auto_splits(int32_t M, int32_t N, int32_t K);
int vllt_gemm_bf16_splitk(const void* A, const void* W, float* C, int32_t M, int32_t N, int32_t K,
                          int32_t splits, void* workspace, int64_t workspace_bytes, int32_t* device_flags,
                          void* stream);

/* ------------------------------------------------------------------------ */
/* Sampling (vllmlite/sampling.py:41-64, vllmlite/speculative.py:86-100)    */
/* ------------------------------------------------------------------------ */

/* Greedy pick per row with the reference's pre-steps: EOS masked to -inf in
 * rows whose eos_mask[r] != 0 (min_tokens, sampling.py:51-52), repetition
 * penalty on the tokens seen by the row (sampling.py:54, seen_bits[r] is a
 * bitmap of ceil(vocab/32) words, may be NULL when penalty[r] == 1), then the
 * first index of the maximum (np.argmax). logits [rows][ld] fp32. */
int vllt_sample_greedy(const float* logits, int32_t rows, int32_t vocab, int32_t ld,
                       const uint8_t* eos_mask, int32_t eos_id, const float* penalty,
                       const uint32_t* seen_bits, int32_t* out_tokens, void* stream);

/* The reference's whole sampler (vllmlite/sampling.py:41-64) for rows with a
 * temperature > 0, one token per row. Row r of the call reads logits row
 * row_index[r] (NULL: row r) of a buffer of logit_rows rows, and applies, in
 * the reference's order: EOS -> -inf where eos_mask[r] != 0 (min_tokens not
 * reached, :51-52), the repetition penalty on the tokens set in seen_bits[r]
 * (ceil(vocab/32) words per row, may be NULL when penalty[r] == 1; :54),
 * division by temperature[r] (:59), top-k (top_k[r] <= 0 or >= vocab keeps
 * all, :16-20), top-p (the nucleus of sampling.py:23-33: descending order,
 * keep while the mass before a token is < top_p[r]) and the draw (:63-64):
 * numpy's Generator.choice given the float64 uniform u[r] it would draw from
 * the request's generator, i.e. the first token whose cumulative kept
 * probability (float64, divided by the total) exceeds u[r]. eos_mask,
 * penalty, seen_bits, top_k and top_p may be NULL (no mask / no penalty /
 * no top-k / top_p = 1). A row_index outside [0, logit_rows) yields -1. */
int vllt_sample_top_p(const float* logits, int32_t rows, int32_t vocab, int32_t ld, int32_t logit_rows,
                      const int32_t* row_index, const uint8_t* eos_mask, int32_t eos_id,
                      const float* penalty, const uint32_t* seen_bits, const float* temperature,
                      const int32_t* top_k, const float* top_p, const double* u, int32_t* out_tokens,
                      void* stream);

/* Speculative accept/reject for a batch of sequences. Sequence s owns logit
 * rows [cu_rows[s], cu_rows[s+1]) = n_drafts[s] + 1 rows (total_rows =
 * cu_rows[num_seqs], passed from the host); drafts are packed at
 * draft_offsets[s]. Writes out_tokens[cu_rows[s] + i] (the emitted tokens)
 * and n_accepted[s]; the number of emitted tokens is n_accepted[s] + 1.
 * Follows verify (vllmlite/speculative.py:86-100). */
int vllt_spec_verify(const float* logits, int32_t ld, int32_t vocab, const int32_t* cu_rows,
                     int32_t total_rows, const int32_t* drafts, const int32_t* draft_offsets,
                     int32_t num_seqs, int32_t* out_tokens, int32_t* n_accepted, void* stream);

/* The accept rule alone over tokens already picked per row (e.g. by
 * vllt_sample_greedy with its EOS mask / penalty): n_accepted[s] = length of
 * the longest prefix where picks[cu_rows[s] + i] == drafts[draft_offsets[s] + i]
 * (speculative.py:92-98). */
int vllt_spec_accept(const int32_t* cu_rows, const int32_t* drafts, const int32_t* draft_offsets,
                     int32_t num_seqs, const int32_t* picks, int32_t* n_accepted, void* stream);

/* ------------------------------------------------------------------------ */
/* Whole forward pass (TinyLlama.forward, vllmlite/model.py:80-120)         */
/* ------------------------------------------------------------------------ */

typedef struct vllt_model_desc {
  /* shape of THIS rank's shard: n_heads, n_kv_heads, d_ff, vocab and
   * vocab_padded are per rank when tp_size > 1 (heads / FFN columns / vocab
   * rows split evenly); d_model, head_dim and embed_rows are global. */
  int32_t n_layers, n_heads, n_kv_heads, head_dim, d_model, d_ff, vocab, vocab_padded;
  int32_t max_seq_len, block_size, num_blocks;
  float rms_eps;
  int32_t dtype;      /* VLLT_F32: fp32 parity path; VLLT_BF16: bf16 weights/activations */
  int32_t tp_size;    /* tensor-parallel ranks (1 = none) */
  int32_t embed_rows; /* rows of tok_emb (the full vocabulary) */
  void* tp_comm;      /* communicator from vllt_tp_init when tp_size > 1 */
  /* weights (device). Per-layer arrays hold n_layers host-side pointers.
   * VLLT_F32 (all fp32, the reference's [in][out] orientation):
   *   wqkv[l]   [d_model][(n_heads + 2*n_kv_heads)*head_dim]  = [wq | wk | wv]
   *   wo[l]     [n_heads*head_dim][d_model]
   *   w_gu[l]   [d_model][2*d_ff], column 2j = w_gate[:, j], 2j+1 = w_up[:, j]
   *   w_down[l] [d_ff][d_model]
   *   lm_head   [d_model][vocab_padded] (zero columns past vocab)
   * VLLT_BF16 (bf16, K-major [out][in] for the tcgen05 GEMM; norms fp32):
   *   wqkv[l]   [(n_heads + 2*n_kv_heads)*head_dim][d_model]  rows [q | k | v]
   *   wo[l]     [d_model][n_heads*head_dim]
   *   w_gu[l]   [2*d_ff][d_model], row 2j = gate_j, 2j+1 = up_j
   *   w_down[l] [d_model][d_ff]
   *   lm_head   [vocab][d_model]  (this rank's vocabulary rows)
   *   tok_emb   [embed_rows][d_model] bf16                                   */
  const void* tok_emb;
  const float* final_norm;
  const void* lm_head;
  const float* rope_cos; /* [max_seq_len][head_dim/2] */
  const float* rope_sin;
  const float* const* attn_norm;
  const void* const* wqkv;
  const void* const* wo;
  const float* const* ffn_norm;
  const void* const* w_gu;
  const void* const* w_down;
  /* KV cache base: [n_layers][num_blocks][n_kv][block_size][head_dim], dtype */
  void* k_cache;
  void* v_cache;
  /* Optional persistent block-table pool [table_pool_slots][caps max_table_width]
   * (device int32). NULL: step records carry their tables; else vllt_forward
   * reads pooled records (see vllt_build_batch_meta_pooled). */
  int32_t* table_pool;
  int32_t table_pool_slots;
  /* Optional token source (device int32 [token_source_len]): the buffer the
   * previous pass's pick kernels wrote; step-record token ids t < 0 read entry
   * -t - 1 of it (see the record layout). The pointer is read when the
   * forward is enqueued, so a CUDA graph keeps it: keep the buffer at one
   * address. NULL: negative ids are errors. */
  const int32_t* token_source;
  int32_t token_source_len;
} vllt_model_desc;

/* Upper bounds of one step, used to size grids (exact counts are read on the
 * device). For eager calls pass the step's own values; a CUDA graph captured
 * with some bounds replays correctly for every step within them. */
typedef struct vllt_step_bounds {
  int32_t tokens;      /* >= T */
  int32_t rows;        /* >= R */
  int32_t decode_seqs; /* >= sequences with a single query token */
  int32_t tiles;       /* >= multi-token query tiles (16 (position, head) rows each) */
  int32_t max_ctx;     /* >= longest context (start + qlen) */
} vllt_step_bounds;

/* Query positions per multi-token attention tile the forward pass uses for
 * this model (the tensor-core prefill kernel takes 128 / n_rep, the generic
 * kernel 16 / n_rep); hosts size vllt_step_bounds.tiles with it. */
int32_t vllt_query_tile_positions(const vllt_model_desc* m);

/* Activation workspace bytes for the given capacities. */
int64_t vllt_forward_workspace_bytes(const vllt_model_desc* m, const vllt_caps* caps);

/* One batched forward pass over a packed step record already on the device:
 * builds the batch metadata into `meta` (see vllt_build_batch_meta), embeds,
 * runs every layer (RMSNorm -> QKV GEMM with RoPE and the K/V cache write
 * fused in its epilogue -> paged attention -> o_proj + residual -> RMSNorm ->
 * gate/up GEMM with SwiGLU -> down + residual), then the final RMSNorm and
 * lm_head on the logit rows only. logits: [max_rows][vocab_padded] fp32;
 * rows >= R are left untouched. With dtype VLLT_BF16 the projections run on
 * the tcgen05 GEMM, the residual stream stays fp32, and with tp_size > 1 the
 * o_proj / down_proj partials are all-reduced (NCCL, bf16) before they join
 * the residual; logits are this rank's vocabulary slice. */
int vllt_forward(const vllt_model_desc* m, const int32_t* step_record, const vllt_caps* caps,
                 const vllt_step_bounds* bounds, void* meta, void* workspace,
                 int64_t workspace_bytes, float* logits, void* stream);

/* ------------------------------------------------------------------------ */
/* Prefix-cache hashing                                                     */
/* ------------------------------------------------------------------------ */

/* Content hashes of full KV blocks, bit-identical to vllm-lite's hash_block
 * (vllmlite/block.py:34-40: blake2b with a 16-byte digest over the previous
 * block's hex digest, "|", and the block's token ids joined by commas,
 * returned as 32 lowercase hex characters), chained block after block as
 * BlockManager.commit and reuse_prefix chain them (block_manager.py:98-120).
 * Chain c (all pointers device memory):
 *   n_blocks[c] full blocks of block_size tokens at tokens + token_offsets[c];
 *   prev_hex (NULL: no chain has one) + 32*c: the hex digest of the block
 *     before the chain, or 32 zero bytes for none (the first block of a
 *     sequence);
 *   out_hex + 32 * (out_offsets[c] + b): the hex digest of block b.
 * The caller keeps every offset inside its buffers. One thread per chain. */
int vllt_prefix_hash_chains(const int32_t* tokens, const int64_t* token_offsets, const int32_t* n_blocks,
                            const int64_t* out_offsets, const uint8_t* prev_hex, int32_t n_chains,
                            int32_t block_size, uint8_t* out_hex, void* stream);

/* ------------------------------------------------------------------------ */
/* Tensor parallelism (bf16 model): NCCL, loaded at run time                */
/* ------------------------------------------------------------------------ */

/* 128-byte communicator id, made on one rank and shared with the others. */
int vllt_tp_unique_id(uint8_t* out128);
/* Join the communicator (call on every rank concurrently, device current). */
int vllt_tp_init(const uint8_t* id128, int32_t rank, int32_t world, void** comm_out);
int vllt_tp_destroy(void* comm);
/* In-place sum over ranks of a bf16 buffer (used between row-parallel layers). */
int vllt_tp_allreduce_bf16(void* buf, int64_t count, void* comm, void* stream);

/* Per logit row: the maximum and the FIRST index of it (np.argmax), index
 * shifted by vocab_offset (this rank's first vocabulary row). Vocab-parallel
 * greedy: each rank reduces its slice, the host or a gather picks the max. */
int vllt_argmax_rows(const float* logits, int32_t rows, int32_t vocab, int32_t ld, int32_t vocab_offset,
                     float* out_val, int32_t* out_idx, void* stream);

#ifdef __cplusplus
}
#endif
#endif /* VLLT_H_ */
