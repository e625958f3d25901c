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
  uint64_t dim2, stride2;        // rank 3: planes, bytes per plane (rank 2: 1, 0)
  uint32_t box2, rank;
};
static_assert(sizeof(HostTensorMap) <= sizeof(CUtensorMap), "map");

inline CUresult encode_tiled(CUtensorMap* m, CUtensorMapDataType dt, cuuint32_t rank, void* base,
                             const cuuint64_t* dims, const cuuint64_t* strides, const cuuint32_t* box,
                             const cuuint32_t* estr, CUtensorMapInterleave, CUtensorMapSwizzle sw,
                             CUtensorMapL2promotion, CUtensorMapFloatOOBfill) {
  const uint32_t esize = dt == CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 ? 2 : dt == CU_TENSOR_MAP_DATA_TYPE_FLOAT32 ? 4 : 1;
  if ((rank != 2 && rank != 3) || !m || !base || (reinterpret_cast<uintptr_t>(base) & 15) || strides[0] % 16 ||
      box[0] == 0 || box[1] == 0 || box[0] > 256 || box[1] > 256 || (box[0] * esize) % 16 || estr[0] != 1 ||
      estr[1] != 1 || (sw == CU_TENSOR_MAP_SWIZZLE_128B && box[0] * esize > 128))
    return CUDA_ERROR_INVALID_VALUE;
  if (rank == 3 && (box[2] == 0 || box[2] > 256 || strides[1] % 16 || estr[2] != 1)) return CUDA_ERROR_INVALID_VALUE;
  HostTensorMap h{static_cast<const unsigned char*>(base), dims[0], dims[1], strides[0], box[0], box[1], esize,
                  (uint32_t)sw, rank == 3 ? dims[2] : 1, rank == 3 ? strides[1] : 0, rank == 3 ? box[2] : 1, rank};
  memset(m, 0, sizeof(*m));
  memcpy(m->opaque, &h, sizeof(h));
  return CUDA_SUCCESS;
}

// One box load at (x, y, z) (z = 0 for a 2-D map); returns the box's bytes
// (the transaction count). The box lands as [box2][box1] rows of box0
// elements; with the 128-byte swizzle, 16-byte chunk c of smem row r goes to
// chunk c ^ (r % 8), which is the address-bit pattern of the device's swizzle
// only for a destination 1024-byte aligned in the shared window: a 128-byte
// swizzled copy into the dynamic shared memory at another offset is reported
// as a launch failure.
inline uint32_t tma_load_host(void* dst, const CUtensorMap* map, int x, int y, int z) {
  HostTensorMap h;
  memcpy(&h, map->opaque, sizeof(h));
  const uint32_t row_bytes = h.box0 * h.esize, rows = h.box1 * h.box2;
  unsigned char* d = static_cast<unsigned char*>(dst);
  const unsigned char* win = dynamic_smem();
  const bool in_window = d >= win && d < win + dynamic_smem_bytes();
  if (((int64_t)x * h.esize) % 16 != 0 ||  // faults on the device: report, copy nothing
      (h.swizzle == CU_TENSOR_MAP_SWIZZLE_128B && in_window && (d - win) % 1024 != 0) ||
      (in_window && (size_t)(d - win) + (size_t)row_bytes * rows > dynamic_smem_bytes())) {
    launch_failed() = true;
    return row_bytes * rows;
  }
  for (uint32_t r = 0; r < rows; ++r)
    for (uint32_t c = 0; c < row_bytes / 16; ++c) {
      const uint32_t at = h.swizzle == CU_TENSOR_MAP_SWIZZLE_128B ? r * row_bytes + ((c ^ (r % 8)) * 16)
                                                                   : r * row_bytes + c * 16;
      const int64_t plane = (int64_t)z + r / h.box1, row = (int64_t)y + r % h.box1;
      const int64_t col = (int64_t)x + (int64_t)c * 16 / h.esize;
      if (plane >= 0 && plane < (int64_t)h.dim2 && row >= 0 && row < (int64_t)h.dim1 && col >= 0 &&
          col < (int64_t)h.dim0)
        memcpy(d + at, h.base + plane * h.stride2 + row * h.stride1 + col * h.esize, 16);
      else
        memset(d + at, 0, 16);
    }
  return row_bytes * rows;
}
inline uint32_t tma_load_2d_host(void* dst, const CUtensorMap* map, int x, int y) {
  return tma_load_host(dst, map, x, y, 0);
}

}  // namespace simt
