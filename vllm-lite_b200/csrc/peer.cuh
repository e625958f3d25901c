// Peer arenas of the fused tensor-parallel all-reduce (small passes).
//
// Arena of rank r (its own device memory, mapped into every rank's process by
// CUDA IPC):
//   [0, 64)     flags[src]  u64, raised by rank src (epoch of its last partial)
//   [256, 264)  epoch base  u64, bumped once per forward by rank r itself
//   [512, ...)  recv[parity][src][T][d] bf16: rank src's partial of all-reduce
//               number i lands in parity i & 1
// All-reduce i of a forward carries the epoch base * 128 + i + 1; flags only
// grow, so nothing is ever reset. Two parities make reuse safe: rank A writes
// parity p of all-reduce i + 2 only after it has seen every rank's flag of
// all-reduce i + 1, which each rank raises after it finished reading
// all-reduce i (stream order).
#pragma once

#include "common.cuh"

namespace vllt {

constexpr int kMaxPeers = 8;
constexpr int64_t kArenaHeader = 512;

inline int64_t peer_arena_bytes(int n, int T, int d) { return kArenaHeader + 2ll * n * T * d * 2; }

struct PeerArena {
  unsigned char* base[kMaxPeers];
  int n, rank, T, d;
  __device__ __forceinline__ unsigned long long* flags(int r) const {
    return reinterpret_cast<unsigned long long*>(base[r]);
  }
  __device__ __forceinline__ unsigned long long* epoch() const {
    return reinterpret_cast<unsigned long long*>(base[rank] + 256);
  }
  __device__ __forceinline__ __nv_bfloat16* recv(int r, int parity, int src) const {
    return reinterpret_cast<__nv_bfloat16*>(base[r] + kArenaHeader) + (int64_t)(parity * n + src) * T * d;
  }
};

// Row-parallel projection epilogue (o_proj, down_proj): this rank's bf16
// partial of rows x 32 columns goes to slot [parity][this rank] of every
// rank's arena (NVLink stores for the peers, plain stores for itself).
struct EpiPushBF16 {
  PeerArena a;
  int parity;
  template <int TN> __device__ void apply(int row, int col, const float (&v)[TN]) const {
    uint4 w[TN / 8];
#pragma unroll
    for (int j = 0; j < TN / 8; ++j) {
      __nv_bfloat162 t0 = __floats2bfloat162_rn(v[8 * j], v[8 * j + 1]);
      __nv_bfloat162 t1 = __floats2bfloat162_rn(v[8 * j + 2], v[8 * j + 3]);
      __nv_bfloat162 t2 = __floats2bfloat162_rn(v[8 * j + 4], v[8 * j + 5]);
      __nv_bfloat162 t3 = __floats2bfloat162_rn(v[8 * j + 6], v[8 * j + 7]);
      w[j].x = *reinterpret_cast<uint32_t*>(&t0); w[j].y = *reinterpret_cast<uint32_t*>(&t1);
      w[j].z = *reinterpret_cast<uint32_t*>(&t2); w[j].w = *reinterpret_cast<uint32_t*>(&t3);
    }
    for (int r = 0; r < a.n; ++r) {
      uint4* dst = reinterpret_cast<uint4*>(a.recv(r, parity, a.rank) + (int64_t)row * a.d + col);
#pragma unroll
      for (int j = 0; j < TN / 8; ++j) dst[j] = w[j];
    }
  }
};

}  // namespace vllt
