// Per-item steps of the device-resident block tables (the pooled step
// record, include/vllt.h), shared by build_meta_kernel and the host-compiled
// tests: plain integer code with no CUDA dependency.
#pragma once

#include <stdint.h>

#ifndef __CUDACC__
#ifndef __host__
#define __host__
#endif
#ifndef __device__
#define __device__
#endif
#endif

namespace vllt {

// Phase 0: one (pool row, table index, block id) update into the pool
// [pool_slots][width]; false, with nothing written, when it lies outside.
__host__ __device__ inline bool pool_update(int32_t* pool, int pool_slots, int width, const int32_t* upd) {
  const int row = upd[0], j = upd[1];
  if (row < 0 || row >= pool_slots || j < 0 || j >= width) return false;
  pool[(int64_t)row * width + j] = upd[2];
  return true;
}

// Phase 2: entry b of a sequence's block table, read through its pool row,
// for a context that uses `used` blocks: -1 past them (never read); -1 with
// *bad set when the row or the block id is out of range.
__host__ __device__ inline int pool_entry(const int32_t* pool, int pool_slots, int width, int row, int b, int used,
                                          int num_blocks, bool* bad) {
  if (b >= used) return -1;
  int blk = -1;
  if (row >= 0 && row < pool_slots) blk = pool[(int64_t)row * width + b];
  if (blk < 0 || blk >= num_blocks) {
    *bad = true;
    return -1;
  }
  return blk;
}

}  // namespace vllt
