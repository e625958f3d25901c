// Test infrastructure: kernels with and without a data race, for the race
// check's self-test (tests/test_race_check_host.py). Each is launched on the
// SIMT emulation of tests/simt_host.h; under ThreadSanitizer the racy ones
// must be reported and the others not.
#include "simt_host.h"
#include "simt_tc.h"

namespace {

// Each thread writes its shared slot, then reads its neighbour's: ordered by
// __syncthreads (correct), or not (a race between two threads of one CTA).
template <bool BARRIER>
__global__ void neighbour_kernel(int* out) {
  __shared__ int slot[64];
  const int t = threadIdx.x;
  slot[t] = t * 3 + (int)blockIdx.x;
  if (BARRIER) __syncthreads();
  out[blockIdx.x * 64 + t] = slot[(t + 1) % 64];
}

// Every CTA adds to one global word: atomically (correct) or with a plain
// read-modify-write (a race between CTAs).
template <bool ATOMIC>
__global__ void count_kernel(int* total) {
  if (threadIdx.x == 0) {
    if (ATOMIC) atomicAdd(total, 1);
    else *total = *total + 1;
  }
}

// A producer warp fills a shared buffer and arrives on an mbarrier; the
// consumer warp waits for the phase (correct) or reads at once (a race that
// only the barrier's happens-before edge can order).
template <bool WAIT>
__global__ void mbarrier_kernel(int* out) {
  __shared__ uint64_t bar;
  __shared__ int buf[32];
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  if (threadIdx.x == 0) simt::tensor::mbar_init(&bar, 32);
  __syncthreads();
  if (warp == 0) {
    buf[lane] = lane + 7;
    simt::tensor::mbar_arrive(&bar);
  } else {
    if (WAIT)
      while (!simt::tensor::mbar_try_wait(&bar, 0)) {
      }
    out[lane] = buf[lane];
  }
}

}  // namespace

extern "C" int race_neighbour(int barrier, int* out) {
  return barrier ? simt::launch(neighbour_kernel<true>, dim3(2), dim3(64), 0, out)
                 : simt::launch(neighbour_kernel<false>, dim3(2), dim3(64), 0, out);
}
extern "C" int race_count(int atomic, int* total) {
  return atomic ? simt::launch(count_kernel<true>, dim3(64), dim3(32), 0, total)
                : simt::launch(count_kernel<false>, dim3(64), dim3(32), 0, total);
}
extern "C" int race_mbarrier(int wait, int* out) {
  return wait ? simt::launch(mbarrier_kernel<true>, dim3(1), dim3(64), 0, out)
              : simt::launch(mbarrier_kernel<false>, dim3(1), dim3(64), 0, out);
}
