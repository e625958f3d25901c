// Paged-attention decode for bf16 caches, head_dim 128, block_size 16.
//
// Same semantics as the generic kernel in attention.cu (paged_attention,
// vllmlite/attention.py:59-98, for one query token per sequence); built for
// the HBM roofline of long-context decode:
//
//   * Staging: every (block, KV head) tile of the cache is 16 rows x 256 B,
//     contiguous. It is fetched with 2-D tensor-map TMA loads (two 16 x 64
//     boxes per tile for K and for V) with the 128-byte swizzle, so the
//     per-token reads of the score loop and the per-column reads of the P.V
//     loop are bank-conflict free without padding. Each warp owns a private
//     2-stage ring (8 KB per stage) guarded by mbarriers; one lane issues the
//     copies, all lanes wait (bounded).
//   * Math: CUDA cores. Scores: lane (token t = lane % 16, half = lane / 16)
//     dots its token's 64-element half with the NREP query heads of the KV
//     group using packed fp32x2 FMAs; the halves are combined with one
//     shuffle. Online softmax in the log2 domain (q pre-scaled by
//     scale * log2 e). P.V: lane owns 4 output columns for all NREP heads.
//   * Work: CTA = (KV head, sequence, split of 64 blocks); 4 warps take the
//     split's blocks round-robin; partial states merge in shared memory, then
//     across splits in the shared merge kernel (natural-log units).
//
// Algorithmic bytes per (token, KV head): 2 * 128 * 2 = 512 B of K and V.

#include <cuda.h>

#include "decode_kernels.cuh"
#include "ops.cuh"

namespace vllt {

namespace {

using namespace dk;

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(f);
  }
  return fn;
}

// 2-D map over a cache laid out [rows][128] bf16, rows = num_blocks * n_kv * 16.
int cache_map(CUtensorMap* m, const void* base, int64_t rows) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) {
    set_error("decode attention: cuTensorMapEncodeTiled unavailable");
    return VLLT_ERR_CUDA;
  }
  VLLT_REQUIRE(((uintptr_t)base & 15) == 0, "decode attention: cache base must be 16-byte aligned");
  const cuuint64_t dims[2] = {(cuuint64_t)kD, (cuuint64_t)rows};
  const cuuint64_t strides[1] = {(cuuint64_t)kD * 2};
  const cuuint32_t box[2] = {64, (cuuint32_t)kBS};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("decode attention: cuTensorMapEncodeTiled failed (%d)", (int)r);
    return VLLT_ERR_CUDA;
  }
  return VLLT_OK;
}

template <int NREP>
int launch_decode(const CUtensorMap& tk, const CUtensorMap& tv, const DecodeParams& p, int items, int splits,
                  cudaStream_t st) {
  const size_t smem = decode_smem<NREP>();
  static PerDeviceOnce smem_opt_in;  // dynamic shared memory above 48 KB, once per device
  smem_opt_in.run([&] {
    cudaFuncSetAttribute(decode_kernel<NREP>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  });
  dim3 grid(p.n_kv, items, splits);
  VLLT_LAUNCH(grid, kWarps * 32, smem, st, decode_kernel<NREP>)(tk, tv, p);
  return check_launch("decode attention");
}

}  // namespace

constexpr int kDecodeSplitBlocks = 64;

// Test injection for the bounded waits (vllt_test_decode_stall): the next
// decode launch of this thread promises the bytes of table index `block` to
// its stage's mbarrier without issuing the copies, and waits at most
// `wait_ns`; every CTA reading that index reports bit 2 and returns.
struct DecodeStall {
  int block = -1;
  uint64_t wait_ns = 0;
};
thread_local DecodeStall g_stall;

int64_t decode_ws_bytes(int P_cap, int H, int max_ctx) {
  const int splits = ceil_div(ceil_div(max_ctx, kBS), kDecodeSplitBlocks);
  return splits <= 1 ? 0 : (int64_t)splits * P_cap * H * (kD + 2) * sizeof(float);
}

bool decode_supported(const AttnCall& c) {
  const int n_rep = c.H / c.n_kv;
  return c.dtype == VLLT_BF16 && c.D == kD && c.bs == kBS && (n_rep == 1 || n_rep == 2 || n_rep == 4 || n_rep == 8);
}

// One single-query item per (sequence); returns VLLT_OK after enqueuing the
// kernel (and the split merge when the context is split).
int decode_pass(const AttnCall& c, const int32_t* item_seq, const int32_t* n_items, int items_cap, int num_seqs,
                int max_ctx, int* err, cudaStream_t st, int (*merge)(const AttnCall&, const int32_t*,
                                                                     const int32_t*, int, int, int, cudaStream_t)) {
  if (items_cap <= 0) return VLLT_OK;
  CUtensorMap tk, tv;
  const int64_t rows = (int64_t)c.num_blocks * c.n_kv * kBS;
  int rc = cache_map(&tk, c.kc, rows);
  if (rc != VLLT_OK) return rc;
  rc = cache_map(&tv, c.vc, rows);
  if (rc != VLLT_OK) return rc;
  DecodeParams p{};
  p.q = reinterpret_cast<const __nv_bfloat16*>(c.q);
  p.out = reinterpret_cast<__nv_bfloat16*>(c.out);
  p.tables = c.tables;
  p.W = c.W;
  p.cu_q = c.cu_q;
  p.ctx = c.ctx;
  p.item_seq = item_seq;
  p.n_items = n_items;
  p.num_seqs = num_seqs;
  p.H = c.H;
  p.n_kv = c.n_kv;
  p.num_blocks = c.num_blocks;
  p.qscale = c.scale * 1.4426950408889634f;
  p.P_cap = c.P_cap;
  p.err = err;
  p.wait_ns = kWaitNs;
  p.stall_block = -1;
  cudaStreamCaptureStatus capturing = cudaStreamCaptureStatusNone;
  if (g_stall.block >= 0 && cudaStreamIsCapturing(st, &capturing) == cudaSuccess &&
      capturing == cudaStreamCaptureStatusNone) {  // one-shot test injection of this thread, eager launches only
    p.stall_block = g_stall.block;
    p.wait_ns = g_stall.wait_ns;
    g_stall.block = -1;
  }
  int splits = ceil_div(ceil_div(max_ctx, kBS), kDecodeSplitBlocks);
  if (splits > 1) {
    const int64_t need = (int64_t)splits * c.P_cap * c.H * (kD + 2) * sizeof(float);
    if (c.ws && c.ws_bytes >= need) {
      p.split_blocks = kDecodeSplitBlocks;
      p.ws_o = c.ws;
      p.ws_ml = c.ws + (int64_t)splits * c.P_cap * c.H * kD;
    } else {
      splits = 1;
    }
  }
  if (!err) {
    set_error("decode attention: error word required");
    return VLLT_ERR_ARG;
  }
  const int n_rep = c.H / c.n_kv;
  switch (n_rep) {
    case 1: rc = launch_decode<1>(tk, tv, p, items_cap, splits, st); break;
    case 2: rc = launch_decode<2>(tk, tv, p, items_cap, splits, st); break;
    case 4: rc = launch_decode<4>(tk, tv, p, items_cap, splits, st); break;
    default: rc = launch_decode<8>(tk, tv, p, items_cap, splits, st); break;
  }
  if (rc != VLLT_OK || splits == 1) return rc;
  return merge(c, item_seq, n_items, items_cap, num_seqs, splits, st);
}

}  // namespace vllt

extern "C" int vllt_test_decode_stall(int32_t table_index, int64_t wait_ns) {
  vllt::clear_error();
  VLLT_REQUIRE(table_index >= 0 && wait_ns > 0 && wait_ns <= 1000000000ll,
               "test_decode_stall: table index >= 0 and 0 < wait_ns <= 1 s");
  vllt::g_stall.block = table_index;
  vllt::g_stall.wait_ns = (uint64_t)wait_ns;
  return VLLT_OK;
}
