// Shared helpers for the vllt CUDA sources (sm_100a only).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <utility>

#include "../../include/vllt.h"

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

__host__ __device__ inline int ceil_div(int a, int b) { return (a + b - 1) / b; }

// ---- element conversion ----------------------------------------------------
__device__ __forceinline__ float to_f32(float x) { return x; }
__device__ __forceinline__ float to_f32(__nv_bfloat16 x) { return __bfloat162float(x); }
template <typename T> __device__ __forceinline__ T from_f32(float x);
template <> __device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) {
  return __float2bfloat16_rn(x);
}

// Four consecutive elements at p (16-byte aligned for float, 8 for bf16) as floats.
__device__ __forceinline__ float4 load4(const float* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ float4 load4(const __nv_bfloat16* p) {
  uint2 u = *reinterpret_cast<const uint2*>(p);
  float4 f;
  f.x = __uint_as_float(u.x << 16);
  f.y = __uint_as_float(u.x & 0xffff0000u);
  f.z = __uint_as_float(u.y << 16);
  f.w = __uint_as_float(u.y & 0xffff0000u);
  return f;
}

// ---- warp reductions -------------------------------------------------------
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// ---- cp.async (16 bytes, L2-only, zero-fill when src_bytes == 0) ------------
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool valid) {
  unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(smem));
  int n = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(gmem), "r"(n));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N> __device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

// Per-thread part of a row argmax over x[0, n) (float, 16-byte aligned),
// threads t, t + nthreads, ... of a block: float4 loads, 8 in flight per
// thread. (bv, bi) keeps the largest value and, among equal values, the
// lowest index (np.argmax's rule); the caller reduces across threads.
__device__ __forceinline__ void row_argmax_part(const float* __restrict__ x, int n, int t, int nthreads, float& bv,
                                                int& bi) {
  auto take = [&](float v, int c) {
    if (v > bv || (v == bv && c < bi)) {
      bv = v;
      bi = c;
    }
  };
  const float4* x4 = reinterpret_cast<const float4*>(x);
  const int n4 = n >> 2;
  int c4 = t;
  for (; c4 + 7 * nthreads < n4; c4 += 8 * nthreads) {
    float4 a[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) a[u] = __ldg(x4 + c4 + u * nthreads);
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int c = 4 * (c4 + u * nthreads);
      take(a[u].x, c); take(a[u].y, c + 1); take(a[u].z, c + 2); take(a[u].w, c + 3);
    }
  }
  for (; c4 < n4; c4 += nthreads) {
    const float4 a = __ldg(x4 + c4);
    const int c = 4 * c4;
    take(a.x, c); take(a.y, c + 1); take(a.z, c + 2); take(a.w, c + 3);
  }
  for (int c = 4 * n4 + t; c < n; c += nthreads) take(x[c], c);
}

// Programmatic dependent launch. A kernel started with launch_pdl may begin
// while the kernel before it on the stream is still running: everything it
// does before pdl_wait() must neither read what earlier kernels write nor
// write anything (barrier set-up, tensor-memory allocation, loads of
// constant weights). pdl_wait() returns once the previous kernel has finished
// and its writes are visible; every thread of a PDL-launched kernel passes it
// before exiting, so its own completion implies its predecessors'.
// pdl_trigger() lets the next PDL-launched kernel start launching now. Both
// are no-ops for kernels launched without the attribute.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

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
