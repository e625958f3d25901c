// Test harness: the device prefix hash (csrc/prefix_hash.cuh) compiled for the
// host, so the CPU suite checks the exact functions the kernel runs against
// the reference's hash_block. Built by tests/test_prefix_hash.py with g++.
#include "prefix_hash.cuh"

extern "C" void hash_chain_host(const uint8_t* prev_hex, const int32_t* tokens, int n_blocks, int block_size,
                                uint8_t* out_hex) {
  vllt::hash_chain(prev_hex, tokens, n_blocks, block_size, out_hex);
}
