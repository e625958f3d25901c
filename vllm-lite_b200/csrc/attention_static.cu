// Paged attention whose scratch memory is a static array owned by the
// library, for callers that cannot allocate device memory themselves.
//
// The device address is looked up once per device and kept for the life of
// the process; it does not survive cudaDeviceReset (a reset context gets a
// new module load), so a caller that resets a device must not call this
// entry point on it again in the same process.
//
// Who needs this: code that runs under a device-memory budget owned by someone
// else (a host framework whose allocator has already claimed the GPU, or a
// process started with a hard memory cap), code that is not allowed to call
// cudaMalloc on its hot path because cudaMalloc may synchronize the device
// and stall a latency-critical decode loop, and plug-ins that receive only
// input and output buffers through a fixed interface. They pass inputs and
// outputs as usual; the split-K partials and the error-flag word live in
// g_attention_scratch below.
//
// The array is file-scope `static __device__`, so every GPU that loads this
// library holds its 16 MiB from module load until the process exits. Host
// code cannot use the symbol itself as a device address: once per device,
// with that device current, cudaGetSymbolAddress gives the real address,
// which is cached and passed to the kernels.

#include <mutex>

#include "ops.cuh"

namespace vllt {

namespace {

constexpr int64_t kStaticScratchBytes = 16ll << 20;  // 16 MiB per device
constexpr int64_t kFlagHeaderBytes = 256;           // first bytes: device error word

static __device__ __align__(256) unsigned char g_attention_scratch[kStaticScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void* g_scratch_addr[kMaxDevices] = {};

// Device address of g_attention_scratch on the current device (set up once).
int scratch_address(void** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    set_error("paged_attention_noalloc: cudaGetDevice failed: %s", cudaGetErrorString(e));
    return VLLT_ERR_CUDA;
  }
  if (dev < 0 || dev >= kMaxDevices) {
    set_error("paged_attention_noalloc: device %d beyond the %d supported", dev, kMaxDevices);
    return VLLT_ERR_UNSUPPORTED;
  }
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_attention_scratch);
    if (e != cudaSuccess || !p) {
      set_error("paged_attention_noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
      return VLLT_ERR_CUDA;
    }
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return VLLT_OK;
}

}  // namespace
}  // namespace vllt

using namespace vllt;

extern "C" int vllt_paged_attention_varlen_noalloc(
    const void* q, const void* k_cache, const void* v_cache, const int32_t* block_tables,
    int32_t table_width, const int32_t* cu_seqlens_q, const int32_t* ctx_lens, int32_t num_seqs,
    int32_t num_tokens, int32_t max_qlen, int32_t max_ctx, int32_t n_heads, int32_t n_kv,
    int32_t head_dim, int32_t block_size, int32_t num_blocks, float scale, int32_t dtype, void* out,
    int32_t* device_flags, void* stream) {
  clear_error();
  VLLT_REQUIRE(num_seqs >= 0 && num_tokens >= 0 && max_qlen >= 0 && max_ctx >= 0 && n_heads > 0 &&
                   n_kv > 0 && n_heads % n_kv == 0 && head_dim > 0 && block_size > 0 &&
                   num_blocks > 0 && table_width > 0,
               "paged_attention_noalloc: bad sizes");
  VLLT_REQUIRE(dtype == VLLT_F32 || dtype == VLLT_BF16, "paged_attention_noalloc: bad dtype");
  const int64_t need = attention_ws_bytes(num_seqs, n_heads, head_dim, max_ctx);
  VLLT_REQUIRE(need <= kStaticScratchBytes,
               "paged_attention_noalloc: this batch needs %lld bytes of scratch; the static scratch "
               "holds %lld (use vllt_paged_attention_varlen with a caller workspace)",
               (long long)need, (long long)kStaticScratchBytes);
  cudaStream_t st = as_stream(stream);
  if (num_seqs == 0 || num_tokens == 0) {  // nothing to attend: report a clean call
    if (device_flags && cudaMemsetAsync(device_flags, 0, sizeof(int32_t), st) != cudaSuccess) {
      set_error("paged_attention_noalloc: clearing the error flags failed");
      return VLLT_ERR_CUDA;
    }
    return VLLT_OK;
  }
  VLLT_REQUIRE(q && k_cache && v_cache && block_tables && cu_seqlens_q && ctx_lens && out,
               "paged_attention_noalloc: null pointer");
  void* scratch = nullptr;
  int rc = scratch_address(&scratch);
  if (rc != VLLT_OK) return rc;
  // the array keeps the previous call's contents: the error word must start at zero
  if (cudaMemsetAsync(scratch, 0, kFlagHeaderBytes, st) != cudaSuccess) {
    set_error("paged_attention_noalloc: clearing the scratch flags failed");
    return VLLT_ERR_CUDA;
  }
  AttnCall c{};
  c.q = q; c.kc = k_cache; c.vc = v_cache; c.out = out;
  c.tables = block_tables; c.W = table_width; c.cu_q = cu_seqlens_q; c.ctx = ctx_lens;
  c.H = n_heads; c.n_kv = n_kv; c.D = head_dim; c.bs = block_size; c.num_blocks = num_blocks;
  c.dtype = dtype; c.scale = scale; c.P_cap = num_seqs;
  c.ws = reinterpret_cast<float*>(scratch);
  c.ws_bytes = kStaticScratchBytes;
  c.err = nullptr;  // the scratch header carries the error word
  c.T_rows = num_tokens;
  rc = attention_pass(c, nullptr, nullptr, nullptr, 0, num_seqs, max_qlen, max_qlen <= 1, max_ctx, st);
  if (rc != VLLT_OK) return rc;
  if (device_flags &&
      cudaMemcpyAsync(device_flags, scratch, sizeof(int32_t), cudaMemcpyDeviceToDevice, st) != cudaSuccess) {
    set_error("paged_attention_noalloc: copying the error flags failed");
    return VLLT_ERR_CUDA;
  }
  return VLLT_OK;
}
