// Prefix-cache content hashes on the device: one thread per sequence chain of
// full KV blocks, each block hashed as vllm-lite's hash_block
// (vllmlite/block.py:34-40) with the previous block's digest chained in
// (vllmlite/block_manager.py:98-120). The arithmetic is in prefix_hash.cuh.

#include "common.cuh"
#include "prefix_hash.cuh"

namespace vllt {

namespace {

__global__ void prefix_hash_kernel(const int32_t* __restrict__ tokens, const int64_t* __restrict__ token_off,
                                   const int32_t* __restrict__ n_blocks, const int64_t* __restrict__ out_off,
                                   const uint8_t* __restrict__ prev_hex, int n_chains, int block_size,
                                   uint8_t* __restrict__ out_hex) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= n_chains) return;
  const int nb = n_blocks[c];
  if (nb <= 0) return;
  hash_chain(prev_hex ? prev_hex + 32 * (int64_t)c : nullptr, tokens + token_off[c], nb, block_size,
             out_hex + 32 * out_off[c]);
}

}  // namespace

}  // namespace vllt

using namespace vllt;

extern "C" int vllt_prefix_hash_chains(const int32_t* tokens, const int64_t* token_offsets, const int32_t* n_blocks,
                                       const int64_t* out_offsets, const uint8_t* prev_hex, int32_t n_chains,
                                       int32_t block_size, uint8_t* out_hex, void* stream) {
  clear_error();
  VLLT_REQUIRE(n_chains >= 0 && block_size > 0 && block_size <= 4096, "prefix_hash: bad sizes");
  if (n_chains == 0) return VLLT_OK;
  VLLT_REQUIRE(tokens && token_offsets && n_blocks && out_offsets && out_hex, "prefix_hash: null pointer");
  const int threads = 128;
  VLLT_LAUNCH(ceil_div(n_chains, threads), threads, 0, as_stream(stream), prefix_hash_kernel)(
      tokens, token_offsets, n_blocks, out_offsets, prev_hex, n_chains, block_size, out_hex);
  return check_launch("prefix_hash");
}
