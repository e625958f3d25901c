// Device helpers shared by the kernels (sm_100a). Kernel headers include
// this file only, so that their code also compiles for the host under a SIMT
// emulation (VLLT_SIMT_HOST, defined by the emulation's build, whose
// cuda_runtime.h / cuda_bf16.h stand-ins come first on the include path; the
// product never defines it): the few helpers written in inline PTX then have
// plain equivalents.
#pragma once

#include <cuda_bf16.h>  // under the host emulation: its stand-in headers
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

// A kernel's dynamic shared memory: `VLLT_DYNAMIC_SMEM(name, align);`
// declares `name` as the unsigned char array of the launch's dynamic shared
// memory, `align`-byte aligned (under the host emulation, the emulation's
// buffer for it). The alignment is a promise the compiler uses: with 1024,
// the run-time rounding of the base to a 1 KB swizzle atom folds away.
#ifdef VLLT_SIMT_HOST
#define VLLT_DYNAMIC_SMEM(name, align) unsigned char* name = ::simt::dynamic_smem()
#else
#define VLLT_DYNAMIC_SMEM(name, align) extern __shared__ __align__(align) unsigned char name[]
#endif

// A kernel launch: `VLLT_LAUNCH(grid, block, smem, stream, kernel)(args...)`
// is `kernel<<<grid, block, smem, stream>>>(args...)` (the kernel last, so a
// template argument list may hold commas); under the host emulation it runs
// the grid there.
#ifdef VLLT_SIMT_HOST
#define VLLT_LAUNCH(grid, block, smem, stream, ...) ::simt::launcher(__VA_ARGS__, grid, block, smem)
#else
#define VLLT_LAUNCH(grid, block, smem, stream, ...) __VA_ARGS__<<<grid, block, smem, stream>>>
#endif

namespace vllt {

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
#ifdef VLLT_SIMT_HOST
inline void cp_async16(void* smem, const void* gmem, bool valid) {
  if (valid) memcpy(smem, gmem, 16); else memset(smem, 0, 16);
}
inline void cp_async_commit() {}
template <int N> inline void cp_async_wait() {}
#else
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool valid) {
  unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(smem));
  int n = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(gmem), "r"(n));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N> __device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}
#endif

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
#ifdef VLLT_SIMT_HOST
inline void pdl_wait() {}
inline void pdl_trigger() {}
#else
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
#endif

}  // namespace vllt
