// Test harness: the temperature sampler of the top_p_kernel
// (csrc/sampler_row.cuh) compiled for the host and run by 256 fibers that
// stand in for the threads of the kernel's CTA (ucontext, one OS thread; a
// barrier hands over to the next fiber, round robin, so every fiber has
// reached it before the first one passes). Each fiber walks the vocabulary as
// threadIdx.x does (c = tid, tid + 256, ...), and every reduction combines the
// threads' partials in the kernel's order (an xor butterfly within each warp of
// 32, then warp 0 over the 8 warp results; IEEE addition is commutative, so
// every lane of a butterfly holds the same bits). The CDF search replays the
// kernel's chunked Hillis-Steele scan in float64 with a carried sum. So the
// float32 sums here are the kernel's sums, and what differs from the device is
// only expf (glibc against CUDA's, a few ulps). Built by the CPU tests with
// g++ (tests/host_build.py).
#include <ucontext.h>

#include <climits>
#include <vector>

#include "sampler_row.cuh"

using namespace vllt::sampler;

namespace {

constexpr int kThreads = 256;  // the kernel's CTA size (sampling.cu)

template <class T, class Op>
T warp_tree(T* v, Op op) {  // __shfl_xor_sync butterfly, offsets 16 .. 1
  for (int o = 16; o > 0; o >>= 1) {
    T nv[32];
    for (int l = 0; l < 32; ++l) nv[l] = op(v[l], v[l ^ o]);
    for (int l = 0; l < 32; ++l) v[l] = nv[l];
  }
  return v[0];
}

template <class T, class Op>
T block_tree(const T* part, Op op, T init) {  // block_reduce of sampling.cu
  T red[32];
  for (int w = 0; w < 32; ++w) {
    T v[32];
    if (w < kThreads / 32) {
      for (int l = 0; l < 32; ++l) v[l] = part[32 * w + l];
      red[w] = warp_tree(v, op);
    } else {
      red[w] = init;
    }
  }
  return warp_tree(red, op);
}

// 256 fibers in lock step. The kernel's control flow is uniform over the CTA
// (every thread meets the same barriers), so a barrier is a hand-over to the
// next fiber: when fiber t runs again, all others are at the same barrier.
struct Fibers {
  ucontext_t main_ctx, ctx[kThreads];
  std::vector<char> stacks;
  int cur = 0, done = 0;
  bool broken = false;  // a fiber finished while another waited at a barrier

  void arrive_and_wait() {
    const int from = cur;
    cur = (cur + 1) % kThreads;
    if (done) {  // non-uniform control flow: stop here
      broken = true;
      swapcontext(&ctx[from], &main_ctx);
    }
    swapcontext(&ctx[from], &ctx[cur]);
  }
  void finish() {  // the fiber's body returned
    const int from = cur;
    if (++done == kThreads) {
      swapcontext(&ctx[from], &main_ctx);
    } else {
      cur = (cur + 1) % kThreads;
      swapcontext(&ctx[from], &ctx[cur]);
    }
  }
};

struct Cta {
  Fibers bar;
  int i32[kThreads];
  float f32[kThreads];
  double f64[kThreads];
  int pick = INT_MAX;
};

struct CtaPolicy {
  Cta* cta;
  int t;
  int tid() const { return t; }
  int stride() const { return kThreads; }

  template <class T, class Op>
  T reduce(T* slots, T v, Op op, T init) {
    slots[t] = v;
    cta->bar.arrive_and_wait();
    const T r = block_tree(slots, op, init);  // every thread reads the same partials
    cta->bar.arrive_and_wait();               // before any slot is written again
    return r;
  }
  int reduce_sum(int v) { return reduce(cta->i32, v, [](int a, int b) { return a + b; }, 0); }
  float reduce_sum(float v) { return reduce(cta->f32, v, [](float a, float b) { return a + b; }, 0.f); }
  double reduce_sum(double v) { return reduce(cta->f64, v, [](double a, double b) { return a + b; }, 0.0); }
  float reduce_max(float v) {
    return reduce(cta->f32, v, [](float a, float b) { return fmaxf(a, b); }, -INFINITY);
  }

  // The kernel's search: chunks of kThreads entries, an inclusive
  // Hillis-Steele scan of each chunk in float64 added to the carried sum, the
  // lowest index of the first chunk that holds the crossing. pc_of is a pure
  // function of c, so thread 0 replays the chunks alone, in the same order.
  template <class F>
  int first_crossing(int n, F pc_of, double u) {
    if (t == 0) {
      double carry = 0.0;
      int pick = INT_MAX;
      for (int base = 0; base < n && pick == INT_MAX; base += kThreads) {
        double pc[kThreads], scan[kThreads];
        for (int i = 0; i < kThreads; ++i) scan[i] = pc[i] = base + i < n ? pc_of(base + i) : 0.0;
        for (int o = 1; o < kThreads; o <<= 1) {
          double nv[kThreads];
          for (int i = 0; i < kThreads; ++i) nv[i] = scan[i] + (i >= o ? scan[i - o] : 0.0);
          for (int i = 0; i < kThreads; ++i) scan[i] = nv[i];
        }
        for (int i = 0; i < kThreads && pick == INT_MAX; ++i) {
          const double cdf = carry + scan[i], prev = cdf - pc[i];
          if (base + i < n && pc[i] > 0.0 && prev <= u && u < cdf) pick = base + i;
        }
        carry += scan[kThreads - 1];
      }
      cta->pick = pick;
    }
    cta->bar.arrive_and_wait();
    const int pick = cta->pick;
    cta->bar.arrive_and_wait();
    return pick == INT_MAX ? -1 : pick;
  }

  template <class F>
  int last(int n, F pred) {
    int best = -1;
    for (int c = t; c < n; c += kThreads)
      if (pred(c)) best = c;
    return reduce(cta->i32, best, [](int a, int b) { return a > b ? a : b; }, -1);
  }
};

}  // namespace

// One row through the kernel's sampler: returns the drawn token and, when
// keep_out is given, the reference's keep set (1 = finite after the EOS mask,
// the penalty, top-k and top-p; tokens already at -inf have probability 0 in
// the draw and are not in it).
extern "C" int sample_row_host(const float* x, int vocab, int mask_eos, int eos_id, float pen, const uint32_t* seen,
                               float temp, int top_k, float top_p, double u, unsigned char* keep_out) {
  RowInput row{x, vocab, mask_eos != 0, eos_id, pen, (seen && pen != 1.f) ? seen : nullptr, temp};
  static Cta cta;  // one OS thread drives the fibers; the harness is not re-entrant
  static std::vector<int> picks(kThreads);
  static std::vector<Thresholds> th(kThreads);
  static struct Job {
    const RowInput* row;
    int top_k;
    float top_p;
    double u;
  } job;
  job = {&row, top_k, top_p, u};
  cta.pick = INT_MAX;
  Fibers& f = cta.bar;
  constexpr size_t kStack = 1 << 16;
  f.stacks.assign(kStack * kThreads, 0);
  f.cur = f.done = 0;
  f.broken = false;
  for (int t = 0; t < kThreads; ++t) {
    getcontext(&f.ctx[t]);
    f.ctx[t].uc_stack.ss_sp = f.stacks.data() + kStack * t;
    f.ctx[t].uc_stack.ss_size = kStack;
    f.ctx[t].uc_link = nullptr;
    makecontext(&f.ctx[t], (void (*)())+[](int t) {
      CtaPolicy pol{&cta, t};
      th[t] = thresholds(pol, *job.row, job.top_k, job.top_p);
      picks[t] = draw(pol, *job.row, th[t], job.u);
      cta.bar.finish();
    }, 1, t);
  }
  swapcontext(&f.main_ctx, &f.ctx[0]);
  if (f.broken) return -3;
  for (int t = 1; t < kThreads; ++t)  // every thread of the CTA agrees (uniform results)
    if (picks[t] != picks[0] || th[t].cut_key != th[0].cut_key || th[t].pmin != th[0].pmin) return -2;
  if (keep_out)
    for (int c = 0; c < vocab; ++c) {
      const float v = row.val(c);
      keep_out[c] = (v > -INFINITY && kept(row, th[0], v)) ? 1 : 0;
    }
  return picks[0];
}
