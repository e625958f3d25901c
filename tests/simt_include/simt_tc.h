// Test infrastructure: the host emulation of the sm_100a instructions the
// library's tensor-core kernels use (gemm_bf16_tc.cuh, attention_prefill_tc.cu),
// so that their own code runs on the SIMT emulation of tests/simt_host.h.
// The kernels' host branches (VLLT_SIMT_HOST) call these functions where the
// device code has inline PTX.
//
//   * mbarriers: a word holds the pending transaction bytes, the pending
//     arrivals, the arrival count and the phase bit; a try_wait that finds
//     the phase incomplete lets the CTA's other threads run;
//   * TMA: a tensor-map load copies its box at once (tests/simt_include/cuda.h)
//     and completes its bytes on the barrier; a test can drop one load, whose
//     bytes then never arrive (the bounded waits must expire);
//   * tensor memory: 128 lanes x 512 columns of 32-bit cells per CTA, filled
//     with NaN at each CTA's start; tcgen05.alloc / dealloc / relinquish are
//     checked (power-of-two column counts from 32 to 512, no allocation after
//     the permit was given up, exactly the allocated ranges freed, nothing
//     held when the CTA exits);
//   * tcgen05.mma.cta_group::1.kind::f16: the instruction descriptor and both
//     shared-memory descriptors are decoded and checked field by field (fp32
//     D, bf16 A and B, no negation or sparsity, M 128, N a multiple of 16 up
//     to 256, version 1, base offset 0, 128-byte swizzle), the operands are
//     read through the descriptors' layouts (K-major: row r, element k at
//     start + (r / 8) * SBO + (r % 8) * 128 + 2k; MN-major B: element (n, k)
//     at start + (n / 64) * LBO + (k / 8) * SBO + (k % 8) * 128 + 2 (n % 64);
//     the 128-byte swizzle then XORs address bits 4-6 with bits 7-9), and
//     D[i][j] = (accumulate ? D : 0) + sum_k A[i][k] B[j][k] is formed at
//     once (products exact, the 16-term sum in double, one rounding to fp32);
//     tcgen05.commit arrives on its barrier at once;
//   * tcgen05.ld / st 32x32b: warp w reaches lanes 32 (w % 4) .. + 31 only;
//     the columns must lie in an allocation;
//   * the %globaltimer that bounds every wait is a virtual clock that moves
//     1 us per reading, so a wait that can never complete expires after a
//     million polls, whatever the host's speed.
// A violation is reported as a launch failure (cudaGetLastError), with a
// line on stderr saying what was violated.
#pragma once

#include <stdint.h>
#include <string.h>

#include <atomic>
#include <cstdio>
#include <vector>

#include "cuda.h"
#include "simt_host.h"

namespace simt {
namespace tensor {

inline void fail(const char* what) {
  std::fprintf(stderr, "simt tensor-core emulation: %s (block %u,%u,%u thread %d)\n", what, ::blockIdx.x,
               ::blockIdx.y, ::blockIdx.z, flat_tid());
  launch_failed() = true;
}

// ---- virtual %globaltimer --------------------------------------------------------
inline uint64_t& clock_state() {
  static thread_local uint64_t t = 0;
  return t;
}
SIMT_INTERNAL inline uint64_t global_ns() { return clock_state() += 1000; }

// ---- mbarrier ------------------------------------------------------------------------
struct MbarWord {
  uint32_t tx;
  uint16_t pending;
  uint8_t expected;
  uint8_t phase;
};
static_assert(sizeof(MbarWord) == 8, "an mbarrier is 8 bytes");
inline MbarWord* word(uint64_t* bar) { return reinterpret_cast<MbarWord*>(bar); }
// The happens-before key of one phase of a barrier (race checking): its
// arrivals and completed copies release it, a wait that sees the phase
// complete acquires it.
inline const char* phase_key(uint64_t* bar, unsigned phase) { return reinterpret_cast<const char*>(bar) + (phase & 1); }
SIMT_INTERNAL inline void settle(MbarWord* m) {
  if (m->pending == 0 && m->tx == 0) {
    m->phase ^= 1;
    m->pending = m->expected;
  }
}
SIMT_INTERNAL inline void mbar_init(uint64_t* bar, unsigned count) {
  if (count == 0 || count > 255) fail("mbarrier.init: arrival count out of the emulated range");
  *word(bar) = MbarWord{0, (uint16_t)count, (uint8_t)count, 0};
}
SIMT_INTERNAL inline void mbar_arrive(uint64_t* bar) {
  MbarWord* m = word(bar);
  hb_release(phase_key(bar, m->phase));
  if (m->pending == 0) fail("mbarrier.arrive: more arrivals than the count");
  --m->pending;
  settle(m);
}
SIMT_INTERNAL inline void mbar_expect_tx(uint64_t* bar, unsigned bytes) {
  word(bar)->tx += bytes;
  mbar_arrive(bar);
}
SIMT_INTERNAL inline bool mbar_try_wait(uint64_t* bar, unsigned parity) {
  if (word(bar)->phase == (parity & 1)) {
    yield();  // the producer of this phase may be another thread of the CTA
    if (word(bar)->phase == (parity & 1)) return false;
  }
  hb_acquire(phase_key(bar, parity));
  return true;
}

// ---- TMA -----------------------------------------------------------------------------
// A test drops the n-th tensor-map load from now on (1: the next one): its
// bytes never reach the barrier.
inline std::atomic<int64_t>& drop_countdown() {
  static std::atomic<int64_t> c{0};
  return c;
}
inline bool dropped() {
  std::atomic<int64_t>& c = drop_countdown();
  if (c.load() <= 0) return false;
  return c.fetch_sub(1) == 1;
}
// The box lands in shared memory as the issuing thread's writes (checked for
// races against the kernel's own accesses), then completes its bytes.
inline void tma_complete(uint64_t* bar, uint32_t bytes);
inline void tma_load(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y, int z) {
  if (dropped()) return;
  tma_complete(bar, tma_load_host(dst, map, x, y, z));
}
SIMT_INTERNAL inline void tma_complete(uint64_t* bar, uint32_t bytes) {
  MbarWord* m = word(bar);
  hb_release(phase_key(bar, m->phase));
  m->tx -= bytes;
  settle(m);
}

// ---- shared-memory addresses ------------------------------------------------------------
// The CTA's shared window is its dynamic shared memory: a shared address is
// the byte offset in it (what the descriptors' 14-bit start fields hold, >> 4).
inline uint32_t saddr(const void* p) {
  const unsigned char* u = static_cast<const unsigned char*>(p);
  const unsigned char* w = dynamic_smem();
  if (u < w || u > w + dynamic_smem_bytes()) {
    fail("shared address of a pointer outside the dynamic shared memory");
    return 0;
  }
  return (uint32_t)(u - w);
}
inline const unsigned char* window_at(uint32_t addr, uint32_t bytes) {
  const uint32_t phys = addr ^ (((addr >> 7) & 7u) << 4);  // 128-byte swizzle on the address bits
  if ((size_t)phys + bytes > dynamic_smem_bytes()) {
    fail("tcgen05.mma: operand outside the dynamic shared memory");
    return nullptr;
  }
  return dynamic_smem() + phys;
}

// ---- tensor memory ----------------------------------------------------------------------
constexpr int kLanes = 128, kCols = 512;
struct Tmem {
  std::vector<uint32_t> cell = std::vector<uint32_t>((size_t)kLanes * kCols);
  uint32_t used = 0;  // bit c: columns [32c, 32c + 32) allocated
  std::vector<std::pair<uint32_t, uint32_t>> allocs;  // (first column, columns)
  bool relinquished = false;
};
inline Tmem& tmem() {
  static thread_local Tmem* t = nullptr;
  if (!t) t = new Tmem;
  return *t;
}
inline void cta_start() {
  Tmem& t = tmem();
  std::fill(t.cell.begin(), t.cell.end(), 0x7FC00000u);  // NaN: a read of unwritten columns shows
  t.used = 0;
  t.allocs.clear();
  t.relinquished = false;
  clock_state() = 0;
}
inline bool cta_exit() {
  if (tmem().used) {
    std::fprintf(stderr, "simt tensor-core emulation: block (%u,%u,%u) exited holding tensor memory\n",
                 ::blockIdx.x, ::blockIdx.y, ::blockIdx.z);
    return false;
  }
  return true;
}
inline const bool hooks_installed = [] {
  cta_start_hook() = &cta_start;
  cta_exit_check() = &cta_exit;
  return true;
}();

inline bool cols_allocated(uint32_t col, uint32_t n) {
  for (const auto& a : tmem().allocs)
    if (col >= a.first && col + n <= a.first + a.second) return true;
  return false;
}

inline int lane_id() { return flat_tid() % 32; }
inline int warp_id() { return flat_tid() / 32; }

// tcgen05.alloc.cta_group::1.sync.aligned: the warp writes the address of
// `ncols` columns (lane 0) to *dst.
inline void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  __syncwarp();
  if (lane_id() == 0) {
    Tmem& t = tmem();
    if (ncols < 32 || ncols > 512 || (ncols & (ncols - 1))) {
      fail("tcgen05.alloc: column count is not a power of two from 32 to 512");
    } else if (t.relinquished) {
      fail("tcgen05.alloc after tcgen05.relinquish_alloc_permit");
    } else {
      const uint32_t chunks = ncols / 32, mask = (chunks >= 32 ? ~0u : ((1u << chunks) - 1));
      bool placed = false;
      for (uint32_t c = 0; c + chunks <= 16 && !placed; c += chunks)
        if (!(t.used & (mask << c))) {
          t.used |= mask << c;
          t.allocs.push_back({c * 32, ncols});
          *dst = c * 32;
          placed = true;
        }
      if (!placed) fail("tcgen05.alloc: not enough free columns (the device would wait forever)");
    }
  }
  __syncwarp();
}
inline void tmem_relinquish() {
  __syncwarp();
  if (lane_id() == 0) tmem().relinquished = true;
  __syncwarp();
}
inline void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  __syncwarp();
  if (lane_id() == 0) {
    Tmem& t = tmem();
    bool found = false;
    for (size_t i = 0; i < t.allocs.size(); ++i)
      if (t.allocs[i].first == taddr && t.allocs[i].second == ncols) {
        const uint32_t chunks = ncols / 32, mask = (chunks >= 32 ? ~0u : ((1u << chunks) - 1));
        t.used &= ~(mask << (taddr / 32));
        t.allocs.erase(t.allocs.begin() + (long)i);
        found = true;
        break;
      }
    if (!found) fail("tcgen05.dealloc of a range that is not an allocation");
  }
  __syncwarp();
}

// tcgen05.ld / st .32x32b.x32: thread t of the warp, TMEM lane (taddr >> 16) + t,
// columns (taddr & 0xffff) .. + 31.
inline uint32_t* tmem_row(uint32_t taddr, int ncols, const char* what) {
  const uint32_t lane0 = taddr >> 16, col = taddr & 0xFFFFu;
  if (lane0 != 32u * (uint32_t)(warp_id() % 4)) {
    fail(what);
    return nullptr;
  }
  if (!cols_allocated(col, (uint32_t)ncols)) {
    fail("tcgen05.ld/st: columns outside every allocation");
    return nullptr;
  }
  return tmem().cell.data() + (size_t)(lane0 + lane_id()) * kCols + col;
}
inline void tmem_ld32(uint32_t taddr, uint32_t* r) {
  __syncwarp();  // .sync.aligned: the whole warp
  const uint32_t* row = tmem_row(taddr, 32, "tcgen05.ld: a warp reads outside its lane quarter");
  for (int i = 0; i < 32; ++i) r[i] = row ? row[i] : 0x7FC00000u;
}
inline void tmem_st32(uint32_t taddr, const uint32_t* r) {
  __syncwarp();
  uint32_t* row = tmem_row(taddr, 32, "tcgen05.st: a warp writes outside its lane quarter");
  if (row)
    for (int i = 0; i < 32; ++i) row[i] = r[i];
}

// ---- tcgen05.mma.cta_group::1.kind::f16 ---------------------------------------------------
struct Desc {
  uint32_t start, lbo, sbo;
};
inline bool decode_desc(uint64_t d, Desc& o) {
  o.start = (uint32_t)(d & 0x3FFF) << 4;
  o.lbo = (uint32_t)((d >> 16) & 0x3FFF) << 4;
  o.sbo = (uint32_t)((d >> 32) & 0x3FFF) << 4;
  if (((d >> 46) & 3) != 1) return fail("smem descriptor: version field is not 1 (sm_100)"), false;
  if (((d >> 49) & 7) != 0) return fail("smem descriptor: nonzero base offset"), false;
  if (((d >> 52) & 1) != 0) return fail("smem descriptor: absolute leading-byte-offset mode"), false;
  if (((d >> 61) & 7) != 2) return fail("smem descriptor: swizzle mode is not 128-byte"), false;
  return true;
}
inline float bf16_at(const unsigned char* p) {
  uint16_t h;
  memcpy(&h, p, 2);
  const uint32_t u = (uint32_t)h << 16;
  float f;
  memcpy(&f, &u, 4);
  return f;
}
// rows x 16 operand elements [row][k] read through a descriptor
inline bool read_operand(const Desc& d, int rows, bool mn_major, float* out) {
  for (int r = 0; r < rows; ++r)
    for (int k = 0; k < 16; ++k) {
      const uint32_t a = mn_major ? d.start + (uint32_t)(r >> 6) * d.lbo + (uint32_t)(k >> 3) * d.sbo +
                                        (uint32_t)(k & 7) * 128 + (uint32_t)(r & 63) * 2
                                  : d.start + (uint32_t)(r >> 3) * d.sbo + (uint32_t)(r & 7) * 128 + (uint32_t)k * 2;
      const unsigned char* p = window_at(a, 2);
      if (!p) return false;
      out[r * 16 + k] = bf16_at(p);
    }
  return true;
}
// tcgen05.mma instructions executed (all threads): tests check the kernels'
// work decomposition against it.
inline std::atomic<int64_t>& mma_count() {
  static std::atomic<int64_t> n{0};
  return n;
}
inline void mma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  ++mma_count();
  if ((idesc & 0xF) != 0) return fail("tcgen05.mma: sparsity or saturation set");
  if (((idesc >> 4) & 3) != 1) return fail("tcgen05.mma: D format is not fp32");
  if (((idesc >> 7) & 7) != 1 || ((idesc >> 10) & 7) != 1) return fail("tcgen05.mma: A or B is not bf16");
  if ((idesc >> 13) & 3) return fail("tcgen05.mma: negated operand");
  if ((idesc >> 15) & 1) return fail("tcgen05.mma: MN-major A (not emulated)");
  if (idesc >> 29) return fail("tcgen05.mma: reserved or shift bits set");
  const bool b_mn = (idesc >> 16) & 1;
  const int N = (int)((idesc >> 17) & 0x3F) << 3, M = (int)((idesc >> 24) & 0x1F) << 4;
  if (M != 128) return fail("tcgen05.mma: M other than 128 (not emulated)");
  if (N < 16 || N > 256 || N % 16) return fail("tcgen05.mma: N not a multiple of 16 in [16, 256]");
  if ((tmem_d >> 16) != 0) return fail("tcgen05.mma: D does not start at lane 0");
  const uint32_t dcol = tmem_d & 0xFFFFu;
  if (!cols_allocated(dcol, (uint32_t)N)) return fail("tcgen05.mma: D columns outside every allocation");
  Desc da, db;
  if (!decode_desc(adesc, da) || !decode_desc(bdesc, db)) return;
  static thread_local std::vector<float> A, B;
  A.resize(128 * 16);
  B.resize((size_t)N * 16);
  if (!read_operand(da, 128, false, A.data()) || !read_operand(db, N, b_mn, B.data())) return;
  uint32_t* cells = tmem().cell.data();
  for (int i = 0; i < 128; ++i) {
    uint32_t* row = cells + (size_t)i * kCols + dcol;
    const float* a = A.data() + i * 16;
    for (int j = 0; j < N; ++j) {
      const float* b = B.data() + j * 16;
      double s = 0.0;
      for (int k = 0; k < 16; ++k) s += (double)a[k] * (double)b[k];  // exact products
      float d = 0.f;
      if (accumulate) memcpy(&d, row + j, 4);
      const float r = (float)((double)d + s);
      memcpy(row + j, &r, 4);
    }
  }
}
// tcgen05.commit ... mbarrier::arrive::one: the MMAs above are complete.
inline void mma_commit(uint64_t* bar) { mbar_arrive(bar); }

// ---- clusters --------------------------------------------------------------------------------
inline uint32_t cluster_rank() { return (uint32_t)::simt::cluster_rank(); }
inline void cluster_sync() { cluster_arrive_wait(); }

// exp2 with the device's flush of results below 2^-126 to zero
inline float ex2_ftz(float x) {
  const float y = exp2f(x);
  return y < 1.17549435e-38f ? 0.f : y;
}

}  // namespace tensor
}  // namespace simt

