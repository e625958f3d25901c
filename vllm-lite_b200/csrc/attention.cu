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

#include "attention_kernels.cuh"
#include "ops.cuh"

namespace vllt {

namespace {

using namespace ak;

template <typename T, int D, int ROWS>
int launch_attention(const AttnParams& p, int grid_items, int splits, cudaStream_t st) {
  const size_t smem = attention_smem_bytes<T, D, ROWS>();
  static PerDeviceOnce smem_opt_in;  // dynamic shared memory above 48 KB, once per device
  smem_opt_in.run([&] {
    cudaFuncSetAttribute(attention_kernel<T, D, ROWS>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)smem);
  });
  dim3 grid(p.n_kv, grid_items, splits);
  VLLT_LAUNCH(grid, kWarps * 32, smem, st, attention_kernel<T, D, ROWS>)(p);
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
    case 8: VLLT_LAUNCH(blocks, 256, 0, st, merge_splits_kernel<T, 8>)(p, splits); break;
    case 16: VLLT_LAUNCH(blocks, 256, 0, st, merge_splits_kernel<T, 16>)(p, splits); break;
    case 32: VLLT_LAUNCH(blocks, 256, 0, st, merge_splits_kernel<T, 32>)(p, splits); break;
    case 48: VLLT_LAUNCH(blocks, 256, 0, st, merge_splits_kernel<T, 48>)(p, splits); break;
    case 64: VLLT_LAUNCH(blocks, 256, 0, st, merge_splits_kernel<T, 64>)(p, splits); break;
    case 128: VLLT_LAUNCH(blocks, 256, 0, st, merge_splits_kernel<T, 128>)(p, splits); break;
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
  // the tensor-core prefill kernel reports through the error word: without one
  // the generic kernel takes the multi-token tiles
  const bool tc_tiles = !single_query && prefill_tc_supported(c) && flags;
  int items_per_seq = 1;
  if (!item_seq) {  // standalone: (sequence, tile) items from the batch shape, tiles of the kernel that runs
    const int qp = single_query ? 1 : tc_tiles ? prefill_tc_positions(n_rep) : tile_positions(n_rep);
    items_per_seq = single_query ? 1 : ceil_div(std::max(max_qlen, 1), qp);
    VLLT_REQUIRE((int64_t)items_per_seq * num_seqs < (1ll << 31), "attention: too many tiles");
    items_cap = items_per_seq * num_seqs;
  } else {  // the metadata builder's tiles are query_tile_positions wide
    VLLT_REQUIRE(single_query || tc_tiles || !prefill_tc_supported(c),
                 "attention: tensor-core query tiles need the error word");
  }
  if (items_cap <= 0) return VLLT_OK;
  if (single_query && decode_supported(c) && flags)
    return decode_pass(c, item_seq, n_items, items_cap, num_seqs, max_ctx, flags, st, merge_decode_splits);
  if (tc_tiles)
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
