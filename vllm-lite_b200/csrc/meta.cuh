// Batch-metadata buffer shared by the meta builder, the attention kernels and
// the forward orchestration (its layout and per-item arithmetic are in
// meta_items.cuh).
#pragma once

#include "common.cuh"
#include "meta_items.cuh"

namespace vllt {

// qp: query positions per multi-token attention tile (see query_tile_positions).
// pool: persistent block-table pool [pool_slots][L.W_cap] for records in the
// pooled layout (NULL for records that carry their tables). token_src: the
// previous pass's picks that negative record token ids refer to (NULL: none);
// vocab: embedding rows every resolved token id must lie below.
int build_batch_meta(const int32_t* rec, const MetaLayout& L, int bs, int num_blocks, int qp,
                     int32_t* meta, cudaStream_t st, int32_t* pool = nullptr, int pool_slots = 0,
                     const int32_t* token_src = nullptr, int token_src_len = 0, int vocab = INT32_MAX);

}  // namespace vllt
