// Test harness: phases 0 and 2 of build_meta_kernel for a pooled step record,
// with the kernel's own per-item code (csrc/table_pool.cuh) compiled for the
// host. Built by tests/test_block_pool.py with g++.
#include "table_pool.cuh"

// Applies the record's updates to `pool` and writes each sequence's table
// [S][W] as the kernel reads it; returns the kernel's error bits.
extern "C" int apply_pooled_host(const int32_t* rec, int32_t* pool, int pool_slots, int width, int block_size,
                                 int num_blocks, int32_t* tables) {
  const int S = rec[0], T = rec[1], W = rec[3], U = rec[4];
  const int32_t* start = rec + 5;
  const int32_t* qlen = start + S;
  const int32_t* slot = qlen + 2 * S + T;  // after counts and tokens
  const int32_t* updates = slot + S;
  int err = 0;
  for (int u = 0; u < U; ++u)
    if (!vllt::pool_update(pool, pool_slots, width, updates + 3 * u)) err |= 2;
  for (int s = 0; s < S; ++s) {
    const int used = (start[s] + qlen[s] + block_size - 1) / block_size;
    for (int b = 0; b < W; ++b) {
      bool bad = false;
      tables[s * W + b] = vllt::pool_entry(pool, pool_slots, width, slot[s], b, used, num_blocks, &bad);
      if (bad) err |= 2;
    }
  }
  return err;
}
