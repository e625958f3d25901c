// Shared helpers for the vllt CUDA sources (sm_100a only).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <utility>

#include "../../include/vllt.h"
#include "device_common.cuh"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "vllt is built for sm_100a (B200) only"
#endif

namespace vllt {

// Thread-local error message behind vllt_last_error().
void set_error(const char* fmt, ...);
void clear_error();

// Maps the last launch / runtime error to VLLT_ERR_CUDA with a message.
int check_launch(const char* what);

#define VLLT_REQUIRE(cond, ...)         \
  do {                                  \
    if (!(cond)) {                      \
      ::vllt::set_error(__VA_ARGS__);   \
      return VLLT_ERR_ARG;              \
    }                                   \
  } while (0)

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// The devices on which one call site's one-time step (a kernel's dynamic
// shared-memory opt-in) has run. Thread-safe: a device is recorded only after
// its step has run, so a concurrent caller either finds it recorded or runs
// the (idempotent) step again; devices from 64 on run it on every call.
class PerDeviceOnce {
 public:
  template <class Fn> void run(Fn&& fn) {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess) dev = -1;
    const bool tracked = dev >= 0 && dev < 64;
    if (tracked && ((done_.load(std::memory_order_acquire) >> dev) & 1ull)) return;
    fn();
    if (tracked) done_.fetch_or(1ull << dev, std::memory_order_acq_rel);
  }

 private:
  std::atomic<uint64_t> done_{0};
};

inline int64_t align_up(int64_t x, int64_t a) { return (x + a - 1) / a * a; }

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace vllt
