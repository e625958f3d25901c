// Test infrastructure: the tensor-map part of the CUDA driver API the library
// uses, for building it for the host on the SIMT emulation (tests/simt_host.h).
// cuTensorMapEncodeTiled checks its arguments as the driver documents them
// (16-byte aligned base and strides, boxes of at most 256 elements per
// dimension whose inner extent is a multiple of 16 bytes, at most 128 bytes
// with the 128-byte swizzle) and records the map; simt::tma_load_2d_host
// copies a box into shared memory with the map's swizzle (16-byte chunk c of
// row r at r * row_bytes + ((c ^ (r % 8)) * 16) for the 128-byte swizzle),
// fills elements outside the tensor with zeros, and treats an x coordinate
// whose byte offset is not a multiple of 16 as a launch failure, since on the
// device that faults.
#pragma once

#include <stdint.h>
#include <string.h>

#include "simt_host.h"

typedef uint32_t cuuint32_t;
typedef uint64_t cuuint64_t;
enum CUresult { CUDA_SUCCESS = 0, CUDA_ERROR_INVALID_VALUE = 1 };
enum CUtensorMapDataType { CU_TENSOR_MAP_DATA_TYPE_UINT8 = 0, CU_TENSOR_MAP_DATA_TYPE_FLOAT32 = 7,
                           CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 = 9 };
enum CUtensorMapInterleave { CU_TENSOR_MAP_INTERLEAVE_NONE = 0 };
enum CUtensorMapSwizzle { CU_TENSOR_MAP_SWIZZLE_NONE = 0, CU_TENSOR_MAP_SWIZZLE_32B = 1, CU_TENSOR_MAP_SWIZZLE_64B = 2,
                          CU_TENSOR_MAP_SWIZZLE_128B = 3 };
enum CUtensorMapL2promotion { CU_TENSOR_MAP_L2_PROMOTION_NONE = 0, CU_TENSOR_MAP_L2_PROMOTION_L2_64B = 1,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_128B = 2, CU_TENSOR_MAP_L2_PROMOTION_L2_256B = 3 };
enum CUtensorMapFloatOOBfill { CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE = 0 };

struct alignas(64) CUtensorMap {
  uint64_t opaque[16];
};

namespace simt {

struct HostTensorMap {  // what the host encoder records in CUtensorMap::opaque
  const unsigned char* base;
  uint64_t dim0, dim1, stride1;  // elements, rows, bytes per row
  uint32_t box0, box1, esize, swizzle;
};
static_assert(sizeof(HostTensorMap) <= sizeof(CUtensorMap), "map");

inline CUresult encode_tiled(CUtensorMap* m, CUtensorMapDataType dt, cuuint32_t rank, void* base,
                             const cuuint64_t* dims, const cuuint64_t* strides, const cuuint32_t* box,
                             const cuuint32_t* estr, CUtensorMapInterleave, CUtensorMapSwizzle sw,
                             CUtensorMapL2promotion, CUtensorMapFloatOOBfill) {
  const uint32_t esize = dt == CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 ? 2 : dt == CU_TENSOR_MAP_DATA_TYPE_FLOAT32 ? 4 : 1;
  if (rank != 2 || !m || !base || (reinterpret_cast<uintptr_t>(base) & 15) || strides[0] % 16 ||
      box[0] == 0 || box[1] == 0 || box[0] > 256 || box[1] > 256 || (box[0] * esize) % 16 || estr[0] != 1 ||
      estr[1] != 1 || (sw == CU_TENSOR_MAP_SWIZZLE_128B && box[0] * esize > 128))
    return CUDA_ERROR_INVALID_VALUE;
  HostTensorMap h{static_cast<const unsigned char*>(base), dims[0], dims[1], strides[0], box[0], box[1], esize,
                  (uint32_t)sw};
  memset(m, 0, sizeof(*m));
  memcpy(m->opaque, &h, sizeof(h));
  return CUDA_SUCCESS;
}

// One 2-D box load at (x, y); returns the box's bytes (the transaction count).
inline uint32_t tma_load_2d_host(void* dst, const CUtensorMap* map, int x, int y) {
  HostTensorMap h;
  memcpy(&h, map->opaque, sizeof(h));
  const uint32_t row_bytes = h.box0 * h.esize;
  if (((int64_t)x * h.esize) % 16 != 0) {  // faults on the device: report, copy nothing
    launch_failed() = true;
    return row_bytes * h.box1;
  }
  unsigned char* d = static_cast<unsigned char*>(dst);
  for (uint32_t r = 0; r < h.box1; ++r)
    for (uint32_t c = 0; c < row_bytes / 16; ++c) {
      const uint32_t at = h.swizzle == CU_TENSOR_MAP_SWIZZLE_128B ? r * row_bytes + ((c ^ (r % 8)) * 16)
                                                                   : r * row_bytes + c * 16;
      const int64_t row = (int64_t)y + r, col = (int64_t)x + (int64_t)c * 16 / h.esize;
      if (row >= 0 && row < (int64_t)h.dim1 && col >= 0 && col < (int64_t)h.dim0)
        memcpy(d + at, h.base + row * h.stride1 + col * h.esize, 16);
      else
        memset(d + at, 0, 16);
    }
  return row_bytes * h.box1;
}

}  // namespace simt
