// Test infrastructure: runs the library's SIMT kernels (plain CUDA C++, no
// inline PTX, no tensor-memory or TMA instructions) on the host, so CPU
// tests can execute the kernels' own code against the oracle.
//
// Each CTA runs as blockDim cooperative fibers on one OS thread (a stack
// switch that saves the callee-saved registers and the FP control words; no
// system call, so a barrier over 256 threads costs microseconds).
// A fiber runs until it reaches a barrier, then hands over to the next
// runnable fiber of the CTA:
//   * __syncthreads() waits for every thread of the CTA that has not exited
//     (threads that returned early no longer count, as on sm_70 and later);
//   * __syncwarp() and the warp shuffles wait for the lanes of the warp that
//     have not exited; a shuffle writes the lane's value to a per-warp slot,
//     waits, reads its source lane's slot and waits again before the slot can
//     be reused;
//   * a barrier that can never complete (threads waiting on different
//     barriers) stops the launch with an error instead of hanging.
// Fibers of one CTA never preempt each other, so their plain loads and stores
// to shared memory are coherent. The CTAs of a launch run at the same time on
// a pool of OS threads (one CTA at a time per thread), as on the GPU's SMs:
// atomics are real read-modify-writes and __threadfence a real fence, and a
// kernel whose CTAs depend on their order or on one another's plain stores
// without them shows it here. __shared__ becomes a static thread_local (one
// instance per OS thread, reused by the CTAs it runs). Math intrinsics map
// to the host's IEEE operations (the _rn forms are exact; approximate ones
// such as __expf or rsqrtf map to the host's expf / 1 / sqrtf, so results
// agree with the device within their stated error, not bit for bit).
//
// Include this before any library header; it defines VLLT_SIMT_HOST, which
// makes the library's device helpers (device_common.cuh) use these shims.
#pragma once

#ifndef VLLT_SIMT_HOST
#define VLLT_SIMT_HOST 1
#endif

#include <algorithm>
#include <sys/mman.h>

#include <climits>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <ctime>
#include <functional>
#include <type_traits>
#include <atomic>
#include <condition_variable>
#include <mutex>
#include <thread>
#include <vector>

// ---- race checking: a build with -fsanitize=thread (tests/test_race_check_host.py) --
// Every emulated GPU thread is a ThreadSanitizer fiber, and the emulation
// states the happens-before edges the hardware gives: a barrier (CTA, warp,
// cluster) orders each participant's accesses before it with every
// participant's accesses after it, an mbarrier phase orders its arrivals and
// completed copies before the waits that see it complete, and a CTA's start
// and end order it against the CTAs an OS thread ran before and after it.
// Shared- and global-memory accesses of the kernels' own code are then
// checked: two threads touching the same bytes, one of them writing, with
// neither ordered before the other, is reported. The emulation's own
// bookkeeping (SIMT_INTERNAL) is not checked.
#if defined(__SANITIZE_THREAD__)
#include <sanitizer/tsan_interface.h>
#define SIMT_INTERNAL __attribute__((no_sanitize("thread"), noinline))
namespace simt {
inline void hb_release(const void* key) { __tsan_release(const_cast<void*>(key)); }
inline void hb_acquire(const void* key) { __tsan_acquire(const_cast<void*>(key)); }
}  // namespace simt
#else
#define SIMT_INTERNAL
namespace simt {
inline void hb_release(const void*) {}
inline void hb_acquire(const void*) {}
}  // namespace simt
#endif

#define __global__
#define __device__
#define __host__
#define __forceinline__ inline
#define __noinline__
#define __launch_bounds__(...)
#define __shared__ static thread_local
#define __align__(n) __attribute__((aligned(n)))
#define __grid_constant__

// ---- vector types ------------------------------------------------------------
struct int2 { int x, y; };
struct alignas(16) int4 { int x, y, z, w; };
struct uint2 { unsigned x, y; };
struct alignas(16) uint4 { unsigned x, y, z, w; };
struct alignas(8) float2 { float x, y; };
struct alignas(16) float4 { float x, y, z, w; };
struct dim3 {
  unsigned x = 1, y = 1, z = 1;
  constexpr dim3() = default;
  constexpr dim3(unsigned a, unsigned b = 1, unsigned c = 1) : x(a), y(b), z(c) {}
};
inline int2 make_int2(int x, int y) { return {x, y}; }
inline int4 make_int4(int x, int y, int z, int w) { return {x, y, z, w}; }
inline uint2 make_uint2(unsigned x, unsigned y) { return {x, y}; }
inline uint4 make_uint4(unsigned x, unsigned y, unsigned z, unsigned w) { return {x, y, z, w}; }
inline float2 make_float2(float x, float y) { return {x, y}; }
inline float4 make_float4(float x, float y, float z, float w) { return {x, y, z, w}; }

// ---- bf16 (storage type and the round-to-nearest-even conversion) ------------
struct __nv_bfloat16 {
  uint16_t bits;
};
inline float __bfloat162float(__nv_bfloat16 h) {
  uint32_t u = (uint32_t)h.bits << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}
inline __nv_bfloat16 __float2bfloat16_rn(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return {(uint16_t)((u >> 16) | 0x40)};  // NaN stays NaN
  u += 0x7fffu + ((u >> 16) & 1u);
  return {(uint16_t)(u >> 16)};
}

struct __nv_bfloat162 {
  __nv_bfloat16 x, y;
};
inline __nv_bfloat162 __floats2bfloat162_rn(float a, float b) { return {__float2bfloat16_rn(a), __float2bfloat16_rn(b)}; }

// ---- scalar intrinsics ---------------------------------------------------------
template <class A, class B> inline typename std::common_type<A, B>::type min(A a, B b) { return b < a ? b : a; }
template <class A, class B> inline typename std::common_type<A, B>::type max(A a, B b) { return a < b ? b : a; }
inline float __fdiv_rn(float a, float b) { return a / b; }
inline float __fmul_rn(float a, float b) { return a * b; }
inline float __fadd_rn(float a, float b) { return a + b; }
inline float __fsub_rn(float a, float b) { return a - b; }
inline float __fmaf_rn(float a, float b, float c) { return std::fmaf(a, b, c); }
inline float __frcp_rn(float a) { return 1.f / a; }
inline float __fsqrt_rn(float a) { return std::sqrt(a); }
inline double __dadd_rn(double a, double b) { return a + b; }
inline float rsqrtf(float a) { return 1.f / std::sqrt(a); }
inline float __expf(float a) { return std::exp(a); }
inline float __logf(float a) { return std::log(a); }
inline float __saturatef(float a) { return a < 0.f ? 0.f : (a > 1.f ? 1.f : a); }
inline uint32_t __float_as_uint(float f) { uint32_t u; std::memcpy(&u, &f, 4); return u; }
inline float __uint_as_float(uint32_t u) { float f; std::memcpy(&f, &u, 4); return f; }
inline int __float_as_int(float f) { int u; std::memcpy(&u, &f, 4); return u; }
inline float __int_as_float(int u) { float f; std::memcpy(&f, &u, 4); return f; }
inline int __clz(int x) { return x == 0 ? 32 : __builtin_clz((unsigned)x); }
inline int __popc(unsigned x) { return __builtin_popcount(x); }
inline int __ffs(int x) { return __builtin_ffs(x); }
template <class T> inline T __ldg(const T* p) { return *p; }
template <class T> inline T __ldcg(const T* p) { return *p; }
template <class T> inline void __stcg(T* p, T v) { *p = v; }
// CTAs run on several OS threads at once: the device-scope fence is a real one
inline void __threadfence() { std::atomic_thread_fence(std::memory_order_seq_cst); }
inline void __threadfence_block() { std::atomic_signal_fence(std::memory_order_seq_cst); }
inline void __nanosleep(unsigned) {}

// packed fp32 pairs (sm_100): element-wise, each rounded once
inline float2 __ffma2_rn(float2 a, float2 b, float2 c) { return {std::fmaf(a.x, b.x, c.x), std::fmaf(a.y, b.y, c.y)}; }
inline float2 __fmul2_rn(float2 a, float2 b) { return {a.x * b.x, a.y * b.y}; }
inline float2 __fadd2_rn(float2 a, float2 b) { return {a.x + b.x, a.y + b.y}; }

// ---- atomics: real read-modify-writes (the CTAs of a cluster run on separate OS threads) --
template <class T, class F> inline T atomic_rmw(T* p, F f) {
  T o;
  __atomic_load(p, &o, __ATOMIC_SEQ_CST);
  T n = f(o);
  while (!__atomic_compare_exchange(p, &o, &n, false, __ATOMIC_SEQ_CST, __ATOMIC_SEQ_CST)) n = f(o);
  return o;
}
template <class T> inline T atomicAdd(T* p, T v) { return atomic_rmw(p, [&](T o) { return (T)(o + v); }); }
template <class T> inline T atomicSub(T* p, T v) { return atomic_rmw(p, [&](T o) { return (T)(o - v); }); }
template <class T> inline T atomicMax(T* p, T v) { return atomic_rmw(p, [&](T o) { return v > o ? v : o; }); }
template <class T> inline T atomicMin(T* p, T v) { return atomic_rmw(p, [&](T o) { return v < o ? v : o; }); }
template <class T> inline T atomicOr(T* p, T v) { return atomic_rmw(p, [&](T o) { return (T)(o | v); }); }
template <class T> inline T atomicAnd(T* p, T v) { return atomic_rmw(p, [&](T o) { return (T)(o & v); }); }
template <class T> inline T atomicExch(T* p, T v) { return atomic_rmw(p, [&](T) { return v; }); }
template <class T> inline T atomicCAS(T* p, T c, T v) { return atomic_rmw(p, [&](T o) { return o == c ? v : o; }); }

// ---- built-in variables: set by the scheduler (threadIdx whenever a fiber resumes) --
// Per OS thread: each thread of the launch pool runs one CTA at a time; the
// CTAs of a thread-block cluster run at the same time, one OS thread each.
inline thread_local dim3 threadIdx, blockIdx, blockDim, gridDim;

// ---- the CTA scheduler ---------------------------------------------------------
namespace simt {

#if !defined(__x86_64__)
#error "the SIMT emulation's context switch is written for x86-64"
#endif

// Saves the callee-saved registers, MXCSR and the x87 control word on the
// current stack, stores the stack pointer in *from, switches to `to` and
// restores the same from there (System V x86-64 ABI).
__attribute__((naked, noinline)) inline void stack_switch(void** /*from*/, void* /*to*/) {
  asm volatile(
      "pushq %rbp\n"
      "pushq %rbx\n"
      "pushq %r12\n"
      "pushq %r13\n"
      "pushq %r14\n"
      "pushq %r15\n"
      "subq $8, %rsp\n"
      "stmxcsr (%rsp)\n"
      "fnstcw 4(%rsp)\n"
      "movq %rsp, (%rdi)\n"
      "movq %rsi, %rsp\n"
      "ldmxcsr (%rsp)\n"
      "fldcw 4(%rsp)\n"
      "addq $8, %rsp\n"
      "popq %r15\n"
      "popq %r14\n"
      "popq %r13\n"
      "popq %r12\n"
      "popq %rbx\n"
      "popq %rbp\n"
      "ret\n");
}

// A fresh stack whose first stack_switch "returns" into entry(), with the
// stack aligned as at a function's entry.
inline void* prepare_stack(char* base, size_t size, void (*entry)()) {
  uintptr_t top = (reinterpret_cast<uintptr_t>(base) + size) & ~uintptr_t(15);
  uint64_t* sp = reinterpret_cast<uint64_t*>(top);
  *--sp = 0;                                    // padding: entry sees rsp % 16 == 8
  *--sp = reinterpret_cast<uint64_t>(entry);    // return address of the first switch
  for (int i = 0; i < 6; ++i) *--sp = 0;        // rbp rbx r12 r13 r14 r15
  uint32_t mxcsr;
  uint16_t fpcw;
  asm volatile("stmxcsr %0" : "=m"(mxcsr));
  asm volatile("fnstcw %0" : "=m"(fpcw));
  *--sp = (uint64_t)mxcsr | ((uint64_t)fpcw << 32);
  return sp;
}

constexpr int kMaxThreads = 1024;
constexpr size_t kStack = 1 << 16;  // per fiber
constexpr int kClusterGroup = -3;   // barrier group of barrier.cluster

struct Fiber {
  void* sp = nullptr;
  dim3 tid;
  int waiting = -2;  // -2 running / runnable, -1 CTA barrier, -3 cluster barrier, w >= 0 warp w's barrier
  bool done = false;
};

struct Cta {
  std::vector<Fiber> f;
  std::vector<char> stacks;
  void* main_sp = nullptr;
  int cur = 0, n = 0, done = 0;
  int live_cta = 0;                  // threads not exited
  int live_warp[kMaxThreads / 32];   // lanes not exited per warp
  int arrived_cta = 0, arrived_cluster = 0;
  int arrived_warp[kMaxThreads / 32];
  uint64_t slot[kMaxThreads / 32][32];  // shuffle exchange
  const std::function<void()>* body = nullptr;
  bool deadlock = false;
  // happens-before keys: barrier groups by generation parity, CTA start / end
  unsigned gen_cta = 0, gen_cluster = 0, gen_warp[kMaxThreads / 32] = {};
  char hb_cta[2], hb_cluster[2], hb_warp[kMaxThreads / 32][2], hb_begin, hb_end;
  std::vector<void*> tsan_fiber;  // the race checker's context per fiber (kept across CTAs)
  void* tsan_main = nullptr;      // and the OS thread's own
};

// The OS threads of one cluster's CTAs: barrier.cluster and the shared-memory
// windows through which a CTA reads its peers' shared memory.
struct Cluster {
  int size = 1;
  std::mutex mu;
  std::condition_variable cv;
  int arrived = 0, finished = 0;
  uint64_t gen = 0;
  bool broken = false;
  std::vector<unsigned char*> dyn;  // per rank: dynamic shared memory
  std::vector<size_t> dyn_bytes;
  std::vector<const char*> anchor;  // per rank: a thread_local of this module (static __shared__ variables)
  char hb[2];                       // happens-before keys of barrier.cluster, by generation parity
};

inline thread_local Cta* tls_cta = nullptr;
// A CTA's dynamic shared memory: a window that ends against a PROT_NONE page,
// so a kernel's access past its dynamic shared memory stops the process as
// the guard pages of the tests' global buffers do. Like the device's shared
// memory it is not cleared between CTAs; each launch fills it with 0xFF bytes
// (a NaN in every float, -1 in every int), so a kernel that reads shared
// memory it never wrote sees it.
struct SmemWindow {
  unsigned char* map = nullptr;
  size_t map_bytes = 0;
  unsigned char* win = nullptr;
  SmemWindow() = default;
  SmemWindow(const SmemWindow&) = delete;
  ~SmemWindow() {
    if (map) munmap(map, map_bytes);
  }
  void prepare(size_t bytes) {
    const size_t page = 4096, data = (bytes + 1023) / 1024 * 1024;
    const size_t need = (data + page - 1) / page * page + page;
    if (need > map_bytes) {
      if (map) munmap(map, map_bytes);
      void* m = mmap(nullptr, need, PROT_READ | PROT_WRITE, MAP_PRIVATE | MAP_ANONYMOUS, -1, 0);
      if (m == MAP_FAILED) std::abort();
      map = static_cast<unsigned char*>(m);
      map_bytes = need;
      if (mprotect(map + map_bytes - page, page, PROT_NONE) != 0) std::abort();
    }
    win = map + map_bytes - page - data;  // 1024-byte aligned: the guard page is page aligned
    std::memset(win, 0xFF, data);
  }
};
inline thread_local SmemWindow* tls_smem = nullptr;
inline thread_local size_t tls_smem_bytes = 0;
inline thread_local Cluster* tls_cluster = nullptr;
inline thread_local int tls_rank = 0;

SIMT_INTERNAL inline Cta& cta() {
  if (!tls_cta) tls_cta = new Cta;
  return *tls_cta;
}
inline uint64_t host_ns() {  // the device's %globaltimer
  timespec t;
  clock_gettime(CLOCK_MONOTONIC, &t);
  return (uint64_t)t.tv_sec * 1000000000ull + (uint64_t)t.tv_nsec;
}
SIMT_INTERNAL inline SmemWindow& dyn_smem() {
  if (!tls_smem) tls_smem = new SmemWindow;
  return *tls_smem;
}
inline const dim3& thread_idx() { return ::threadIdx; }
inline unsigned char* dynamic_smem() { return dyn_smem().win; }  // 1024-byte aligned
inline size_t dynamic_smem_bytes() { return tls_smem_bytes; }
// A thread_local of this module: static __shared__ variables (thread_local
// here) sit at the same offset from it in every OS thread's block of the
// module's thread-local storage. (Host builds pass -fno-gnu-unique, so that a
// module's inline and template statics stay its own when several modules
// that compiled the same kernels are loaded.)
__attribute__((visibility("hidden"))) inline thread_local char tls_anchor_byte;
inline const char* tls_anchor() { return &tls_anchor_byte; }

// Tells the race checker which context runs next (fiber i, or -1: the OS
// thread's CTA scheduler), right before the stack switch; no happens-before.
SIMT_INTERNAL inline void to_context(Cta& c, int i) {
#if defined(__SANITIZE_THREAD__)
  __tsan_switch_to_fiber(i < 0 ? c.tsan_main : c.tsan_fiber[i], __tsan_switch_to_fiber_no_sync);
#else
  (void)c;
  (void)i;
#endif
}

SIMT_INTERNAL inline void switch_next() {
  Cta& c = cta();
  const int from = c.cur;
  for (int k = 1; k <= c.n; ++k) {
    const int i = (from + k) % c.n;
    if (!c.f[i].done && c.f[i].waiting == -2) {
      if (i == from) return;
      c.cur = i;
      void** save = &c.f[from].sp;  // no access of the CTA's state between the
      void* to = c.f[i].sp;         // race checker's context switch and the stack's
      to_context(c, i);
      stack_switch(save, to);
      ::threadIdx = c.f[c.cur].tid;  // resumed: this fiber's index again
      return;
    }
  }
  // nobody can run: every live thread waits on a barrier that cannot complete
  c.deadlock = true;
  void** save = &c.f[from].sp;
  to_context(c, -1);
  stack_switch(save, c.main_sp);
}

// Let the other runnable threads of the CTA run (a spin-wait's iteration).
inline void yield() { switch_next(); }

// Schedule variation: with a nonzero seed, a released barrier and the start
// of a CTA hand over to a pseudo-random runnable thread instead of letting
// the releasing one continue, so reads that race with another thread's writes
// between two barriers see different orders from run to run of the seed.
inline uint64_t& schedule_seed() {
  static thread_local uint64_t s = 0;
  return s;
}
SIMT_INTERNAL inline uint32_t next_random() {
  uint64_t& x = schedule_seed();
  x ^= x << 13;
  x ^= x >> 7;
  x ^= x << 17;
  return (uint32_t)(x >> 32);
}

inline void switch_to(int i);

SIMT_INTERNAL inline void release(int group) {
  Cta& c = cta();
  for (auto& fb : c.f)
    if (!fb.done && fb.waiting == group) fb.waiting = -2;
  if (group == -1) c.arrived_cta = 0, ++c.gen_cta;
  else if (group == kClusterGroup) c.arrived_cluster = 0, ++c.gen_cluster;
  else c.arrived_warp[group] = 0, ++c.gen_warp[group];
}

// The happens-before key of the current generation of a barrier group.
SIMT_INTERNAL inline const char* hb_key(Cta& c, int group) {
  if (group == -1) return &c.hb_cta[c.gen_cta & 1];
  if (group == kClusterGroup) return &c.hb_cluster[c.gen_cluster & 1];
  return &c.hb_warp[group][c.gen_warp[group] & 1];
}

SIMT_INTERNAL inline void handover() {  // after a release: a random runnable thread continues
  Cta& c = cta();
  if (!schedule_seed()) return;
  const int pick = (int)(next_random() % (uint32_t)c.n);
  for (int k = 0; k < c.n; ++k) {
    const int i = (pick + k) % c.n;
    if (!c.f[i].done && c.f[i].waiting == -2) {
      switch_to(i);
      break;
    }
  }
}

SIMT_INTERNAL inline void arrive(int group) {  // -1: the CTA; w: warp w
  Cta& c = cta();
  const char* key = hb_key(c, group);
  hb_release(key);
  int& arrived = group < 0 ? c.arrived_cta : c.arrived_warp[group];
  const int size = group < 0 ? c.live_cta : c.live_warp[group];
  if (++arrived >= size) {
    release(group);
    handover();
    hb_acquire(key);
    return;
  }
  c.f[c.cur].waiting = group;
  switch_next();
  hb_acquire(key);
}

// The cluster-wide half of barrier.cluster, once every live thread of this
// CTA has arrived: waits (blocking this OS thread) for the other CTAs of the
// cluster. False if it can never complete (a peer CTA exited, or a peer's
// threads deadlocked).
SIMT_INTERNAL inline bool cluster_os_barrier() {
  Cluster* cl = tls_cluster;
  if (!cl || cl->size == 1) return true;
  std::unique_lock<std::mutex> lk(cl->mu);
  if (cl->broken || cl->finished > 0) {
    cl->broken = true;
    cl->cv.notify_all();
    return false;
  }
  const uint64_t g = cl->gen;
  if (++cl->arrived == cl->size) {
    cl->arrived = 0;
    ++cl->gen;
    cl->cv.notify_all();
    return true;
  }
  cl->cv.wait(lk, [&] { return cl->gen != g || cl->broken; });
  return cl->gen != g;
}

SIMT_INTERNAL inline void complete_cluster_barrier() {
  Cta& c = cta();
  if (!cluster_os_barrier()) {  // the launch fails: back to the CTA's scheduler
    c.deadlock = true;
    void** save = &c.f[c.cur].sp;
    to_context(c, -1);
    stack_switch(save, c.main_sp);
  }
  release(kClusterGroup);
}

// barrier.cluster.arrive + barrier.cluster.wait (a CTA barrier without a cluster).
SIMT_INTERNAL inline void cluster_arrive_wait() {
  Cta& c = cta();
  // one key for every thread of the cluster: the OS-level barrier lets no
  // thread past before all have arrived (and released)
  const char* key = tls_cluster && tls_cluster->size > 1 ? &tls_cluster->hb[tls_cluster->gen & 1]
                                                         : hb_key(c, kClusterGroup);
  hb_release(key);
  if (++c.arrived_cluster >= c.live_cta) {
    complete_cluster_barrier();
    handover();
    hb_acquire(key);
    return;
  }
  c.f[c.cur].waiting = kClusterGroup;
  switch_next();
  hb_acquire(key);
}

// Run thread i now; the current thread stays runnable and resumes later.
SIMT_INTERNAL inline void switch_to(int i) {
  Cta& c = cta();
  const int from = c.cur;
  if (i == from) return;
  c.cur = i;
  void** save = &c.f[from].sp;
  void* to = c.f[i].sp;
  to_context(c, i);
  stack_switch(save, to);
  ::threadIdx = c.f[c.cur].tid;
}

SIMT_INTERNAL inline void exit_thread() {
  Cta& c = cta();
  Fiber* f = c.f.data();
  Fiber& me = f[c.cur];
  me.done = true;
  ++c.done;
  const int w = (int)((me.tid.z * ::blockDim.y + me.tid.y) * ::blockDim.x + me.tid.x) / 32;
  --c.live_cta;
  --c.live_warp[w];
  if (c.arrived_cta > 0 && c.arrived_cta >= c.live_cta) release(-1);
  if (c.arrived_warp[w] > 0 && c.arrived_warp[w] >= c.live_warp[w]) release(w);
  if (c.arrived_cluster > 0 && c.arrived_cluster >= c.live_cta) complete_cluster_barrier();
  // next: another runnable thread, else (the last thread, or every thread left
  // waits on a barrier that cannot complete) the CTA's scheduler
  int next = -1;
  for (int k = 1; c.done < c.n && k <= c.n && next < 0; ++k) {
    const int i = (c.cur + k) % c.n;
    if (!f[i].done && f[i].waiting == -2) next = i;
  }
  if (next < 0 && c.done < c.n) c.deadlock = true;
  void** save = &me.sp;
  void* to = next < 0 ? c.main_sp : f[next].sp;
#if defined(__SANITIZE_THREAD__)
  void* ctx = next < 0 ? c.tsan_main : c.tsan_fiber.data()[next];
#endif
  if (next >= 0) c.cur = next;
  // This thread's last access of the CTA's state: the scheduler's acquire of
  // hb_end at the CTA's end then orders all of them before what follows.
  hb_release(&c.hb_end);
#if defined(__SANITIZE_THREAD__)
  __tsan_switch_to_fiber(ctx, __tsan_switch_to_fiber_no_sync);
#endif
  stack_switch(save, to);  // never resumed
}

SIMT_INTERNAL inline void trampoline() {
  hb_acquire(&cta().hb_begin);
  ::threadIdx = cta().f[cta().cur].tid;
  (*cta().body)();
  exit_thread();
}

inline int flat_tid() {
  const dim3& t = thread_idx();
  return (int)((t.z * ::blockDim.y + t.y) * ::blockDim.x + t.x);
}

// Checks a CTA's state when it has finished (tensor memory, ...): set by the
// tensor-core emulation; false fails the launch.
inline bool (*&cta_exit_check())() {
  static bool (*f)() = nullptr;
  return f;
}
inline void (*&cta_start_hook())() {
  static void (*f)() = nullptr;
  return f;
}

// Runs CTA `bid` (every thread of it) on this OS thread; false if its threads
// waited on barriers that could never complete.
SIMT_INTERNAL inline bool run_cta(dim3 bid, dim3 block, const std::function<void()>& body) {
  const int n = (int)(block.x * block.y * block.z);
  ::blockIdx = bid;
  Cta& c = cta();
  if (c.stacks.size() < kStack * n) c.stacks.resize(kStack * n);
  c.f.assign(n, Fiber{});
  c.n = n;
  c.cur = c.done = 0;
  c.live_cta = n;
  c.arrived_cta = c.arrived_cluster = 0;
  for (int w = 0; w < kMaxThreads / 32; ++w) {
    c.live_warp[w] = std::max(0, std::min(32, n - 32 * w));
    c.arrived_warp[w] = 0;
  }
  c.body = &body;
  c.deadlock = false;
  for (int i = 0; i < n; ++i) {
    c.f[i].tid = dim3(i % block.x, (i / block.x) % block.y, i / (block.x * block.y));
    c.f[i].sp = prepare_stack(c.stacks.data() + kStack * i, kStack, trampoline);
  }
#if defined(__SANITIZE_THREAD__)
  c.tsan_main = __tsan_get_current_fiber();
  while ((int)c.tsan_fiber.size() < n) c.tsan_fiber.push_back(__tsan_create_fiber(0));
#endif
  if (cta_start_hook()) cta_start_hook()();
  hb_release(&c.hb_begin);
  c.cur = schedule_seed() ? (int)(next_random() % (uint32_t)n) : 0;
  void* first = c.f[c.cur].sp;
  to_context(c, c.cur);
  stack_switch(&c.main_sp, first);
  hb_acquire(&c.hb_end);
  if (c.deadlock) {
    std::fprintf(stderr, "simt: block (%u,%u,%u): threads wait on barriers that cannot complete\n", bid.x, bid.y,
                 bid.z);
    return false;
  }
  if (cta_exit_check() && !cta_exit_check()()) return false;
  return true;
}

inline void set_smem(size_t smem) {
  dyn_smem().prepare(smem);
  tls_smem_bytes = smem;
}

// Worker OS threads that run the CTAs of a launch at the same time, as the
// SMs do: each takes the next CTA index until the grid is done (one CTA at a
// time per OS thread, its fibers cooperative). VLLT_SIMT_THREADS sets their
// number (1: every CTA on the launching thread, in index order); by default
// one per host core, at most 32. The pool lives until the process exits.
struct GridPool {
  std::mutex mu, launch_mu;
  std::condition_variable go, idle;
  const std::function<void()>* job = nullptr;
  uint64_t gen = 0;
  int busy = 0, workers = 0;
};
inline int pool_size() {
  static const int n = [] {
    const char* e = std::getenv("VLLT_SIMT_THREADS");
    int v = e ? std::atoi(e) : (int)std::thread::hardware_concurrency();
    return std::max(1, std::min(v, 32));
  }();
  return n;
}
inline GridPool& grid_pool() {
  static GridPool* p = [] {
    GridPool* g = new GridPool;  // never destroyed: the workers wait on it until exit
    g->workers = pool_size() - 1;
    for (int w = 0; w < g->workers; ++w)
      std::thread([g] {
        uint64_t seen = 0;
        for (;;) {
          const std::function<void()>* job;
          {
            std::unique_lock<std::mutex> lk(g->mu);
            g->go.wait(lk, [&] { return g->gen != seen; });
            seen = g->gen;
            job = g->job;
          }
          (*job)();
          std::lock_guard<std::mutex> lk(g->mu);
          if (--g->busy == 0) g->idle.notify_all();
        }
      }).detach();
    return g;
  }();
  return *p;
}

// Runs body() as every thread of every CTA of the grid; returns false if a
// CTA's threads waited on barriers that could never complete. Without a
// cluster, the grid's CTAs are spread over the pool's OS threads; each CTA's
// shuffled schedule (a nonzero seed) is seeded from the launch's seed and the
// CTA's index, so it does not depend on which thread runs it. With a cluster
// of `cluster` CTAs along x, the CTAs of one cluster run at the same time,
// each on its own OS thread, and clusters one after another.
// A B200 CTA can have at most 227 KB of dynamic shared memory (opted in),
// grids at most 2^31 - 1 CTAs along x and 65,535 along y and z.
constexpr size_t kMaxDynamicSmem = 227 * 1024;

inline bool run_grid(dim3 grid, dim3 block, size_t smem, const std::function<void()>& body, unsigned cluster = 1) {
  const int n = (int)(block.x * block.y * block.z);
  if (n < 1 || n > kMaxThreads || cluster < 1 || grid.x % cluster) return false;
  if (smem > kMaxDynamicSmem || grid.y > 65535 || grid.z > 65535 || grid.x > 2147483647u) {
    std::fprintf(stderr, "simt: launch of %u x %u x %u CTAs with %zu bytes of dynamic shared memory exceeds the "
                 "device's limits\n", grid.x, grid.y, grid.z, smem);
    return false;
  }
  ::gridDim = grid;
  ::blockDim = block;
  const uint64_t seed = schedule_seed();
  if (cluster == 1) {
    const int64_t n_cta = (int64_t)grid.x * grid.y * grid.z;
    std::atomic<int64_t> next{0};
    std::atomic<bool> ok{true};
    const std::function<void()> job = [&] {
      ::gridDim = grid;
      ::blockDim = block;
      set_smem(smem);
      for (int64_t i; ok.load() && (i = next.fetch_add(1)) < n_cta;) {
        const dim3 bid((unsigned)(i % grid.x), (unsigned)(i / grid.x % grid.y), (unsigned)(i / grid.x / grid.y));
        schedule_seed() = seed ? seed ^ (0x9E3779B97F4A7C15ull * (uint64_t)(i + 1)) : 0;
        if (!run_cta(bid, block, body)) ok = false;
      }
    };
    GridPool& g = grid_pool();
    const int helpers = (int)std::min<int64_t>(g.workers, n_cta - 1);
    if (helpers <= 0) {
      job();
    } else {
      std::lock_guard<std::mutex> one_launch(g.launch_mu);
      {
        std::lock_guard<std::mutex> lk(g.mu);
        g.job = &job;
        g.busy = g.workers;
        ++g.gen;
      }
      g.go.notify_all();
      job();
      std::unique_lock<std::mutex> lk(g.mu);
      g.idle.wait(lk, [&] { return g.busy == 0; });
    }
    schedule_seed() = seed;
    return ok.load();
  }
  for (unsigned bz = 0; bz < grid.z; ++bz)
    for (unsigned by = 0; by < grid.y; ++by)
      for (unsigned cx = 0; cx < grid.x / cluster; ++cx) {
        Cluster cl;
        cl.size = (int)cluster;
        cl.dyn.assign(cluster, nullptr);
        cl.dyn_bytes.assign(cluster, 0);
        cl.anchor.assign(cluster, nullptr);
        std::vector<char> ok(cluster, 0);
        std::vector<std::thread> th;
        for (unsigned r = 0; r < cluster; ++r)
          th.emplace_back([&, r] {
            ::gridDim = grid;
            ::blockDim = block;
            tls_cluster = &cl;
            tls_rank = (int)r;
            schedule_seed() = seed ? seed ^ (0x9E3779B97F4A7C15ull * (r + 1)) : 0;
            set_smem(smem);
            {
              std::lock_guard<std::mutex> lk(cl.mu);
              cl.dyn[r] = dynamic_smem();
              cl.dyn_bytes[r] = smem;
              cl.anchor[r] = tls_anchor();
            }
            if (cluster_os_barrier()) ok[r] = run_cta(dim3(cx * cluster + r, by, bz), block, body);
            {
              std::lock_guard<std::mutex> lk(cl.mu);
              ++cl.finished;
              if (!ok[r] || cl.arrived > 0) cl.broken = true;
              cl.cv.notify_all();
            }
            delete tls_cta;
            tls_cta = nullptr;
            delete tls_smem;
            tls_smem = nullptr;
            tls_cluster = nullptr;
          });
        for (auto& t : th) t.join();
        for (unsigned r = 0; r < cluster; ++r)
          if (!ok[r]) return false;
      }
  return true;
}

// The rank of this CTA in its cluster (%cluster_ctarank).
inline int cluster_rank() { return tls_cluster ? tls_rank : 0; }

// A pointer into this CTA's shared memory (dynamic, or a static __shared__
// variable) as the same location in CTA `rank` of the cluster (mapa).
inline void* map_shared(const void* p, int rank) {
  Cluster* cl = tls_cluster;
  if (!cl || rank == tls_rank) return const_cast<void*>(p);
  const unsigned char* u = static_cast<const unsigned char*>(p);
  unsigned char* base = dynamic_smem();
  if (u >= base && u < base + tls_smem_bytes) return cl->dyn[rank] + (u - base);
  return const_cast<char*>(cl->anchor[rank]) + (static_cast<const char*>(p) - tls_anchor());
}

template <class... KArgs, class... Args>
inline bool launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, Args... args) {
  std::function<void()> body = [&] { kernel(args...); };
  return run_grid(grid, block, smem, body);
}
template <class... KArgs, class... Args>
inline bool launch_cluster(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, unsigned cluster,
                           Args... args) {
  std::function<void()> body = [&] { kernel(args...); };
  return run_grid(grid, block, smem, body, cluster);
}

// Sticky launch error (a barrier that could not complete, a fault the
// emulation detects), read and cleared by the emulated cudaGetLastError.
inline std::atomic<bool>& launch_failed() {
  static std::atomic<bool> f{false};
  return f;
}

// VLLT_LAUNCH(grid, block, smem, stream, kernel)(args...) under the emulation.
template <class... KArgs>
struct Launcher {
  void (*kernel)(KArgs...);
  dim3 grid, block;
  size_t smem;
  template <class... Args>
  void operator()(Args&&... args) const {
    if (!launch(kernel, grid, block, smem, static_cast<KArgs>(args)...)) launch_failed() = true;
  }
};
template <class... KArgs>
inline Launcher<KArgs...> launcher(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem) {
  return {kernel, grid, block, smem};
}

template <class T>
SIMT_INTERNAL inline T shfl(T v, int src_lane, bool in_range) {
  static_assert(sizeof(T) <= 8, "shuffle of more than 8 bytes");
  Cta& c = cta();
  const int t = flat_tid(), w = t / 32, lane = t % 32;
  uint64_t u = 0;
  std::memcpy(&u, &v, sizeof(T));
  c.slot[w][lane] = u;
  arrive(w);
  T r = v;
  if (in_range) std::memcpy(&r, &c.slot[w][src_lane], sizeof(T));
  arrive(w);
  return r;
}

}  // namespace simt


inline void __syncthreads() { simt::arrive(-1); }
SIMT_INTERNAL inline int __syncthreads_or(int p) {
  static thread_local int acc;
  simt::arrive(-1);
  acc = 0;
  simt::arrive(-1);
  if (p) acc = 1;
  simt::arrive(-1);
  const int r = acc;
  simt::arrive(-1);
  return r;
}
inline void __syncwarp(unsigned = 0xffffffffu) { simt::arrive(simt::flat_tid() / 32); }
template <class T> inline T __shfl_xor_sync(unsigned, T v, int o, int = 32) {
  const int lane = simt::flat_tid() % 32;
  return simt::shfl(v, lane ^ o, true);
}
template <class T> inline T __shfl_sync(unsigned, T v, int src, int = 32) { return simt::shfl(v, src & 31, true); }
template <class T> inline T __shfl_down_sync(unsigned, T v, unsigned d, int = 32) {
  const int lane = simt::flat_tid() % 32;
  return simt::shfl(v, lane + (int)d, lane + (int)d < 32);
}
template <class T> inline T __shfl_up_sync(unsigned, T v, unsigned d, int = 32) {
  const int lane = simt::flat_tid() % 32;
  return simt::shfl(v, lane - (int)d, lane - (int)d >= 0);
}
SIMT_INTERNAL inline unsigned __ballot_sync(unsigned, int p) {
  simt::Cta& c = simt::cta();
  const int t = simt::flat_tid(), w = t / 32, lane = t % 32;
  c.slot[w][lane] = p ? 1 : 0;
  simt::arrive(w);
  unsigned r = 0;
  for (int o = 0; o < c.live_warp[w] && o < 32; ++o)
    if (c.slot[w][o]) r |= 1u << o;
  simt::arrive(w);
  return r;
}
inline int __all_sync(unsigned m, int p) { return __ballot_sync(m, !p) == 0; }
inline int __any_sync(unsigned m, int p) { return __ballot_sync(m, p) != 0; }
