// Host build of rusttorch_b200/csrc/rt_libm.cuh, compared with this
// machine's glibc (the reference's libm).  Test infrastructure: built and
// loaded by tests/test_libm_restatement.py.
#include <math.h>
#include <stdint.h>
#include <string.h>

#include <thread>
#include <vector>

#include "../../rusttorch_b200/csrc/rt_libm.cuh"
#include "../../rusttorch_b200/csrc/rt_ops.cuh"

static float ref(int which, float x) {
  switch (which) {
    case 0: return expf(x);
    case 1: return expm1f(x);
    case 2: return tanhf(x);
    case 3: return logf(x);
    case 5: return expf(x);                  // 5: expf_glibc_nonpos (x <= 0, NaN)
    case 6: return (float)log((double)x);    // 6: logf_pos (positive normals, NaN)
    case 7: return tanhf(x);                 // 7: tanhf_glibc_ge1 (1 <= |x| < 22)
    default: return (float)log((double)x);   // 4: logf_tab against a double log
  }
}

static float mine(int which, float x) {
  switch (which) {
    case 0: return rt::expf_glibc(x);
    case 1: return rt::expm1f_glibc(x);
    case 2: return rt::tanhf_glibc(x);
    case 3: return rt::logf_cr(x);
    case 5: return rt::expf_glibc_nonpos(x);
    case 6: return rt::logf_pos(x);
    case 7: return rt::tanhf_glibc_ge1(x);
    default: return rt::logf_tab(x);
  }
}

// Counts inputs u = start, start+stride, ... < stop whose result bits differ
// (any two NaNs compare equal).  *first_bad receives the first such input.
extern "C" uint64_t libm_mismatches(int which, uint64_t start, uint64_t stop, uint64_t stride,
                                    int threads, uint32_t* first_bad) {
  if (threads < 1) threads = 1;
  std::vector<uint64_t> bad(threads, 0);
  std::vector<uint64_t> first(threads, UINT64_MAX);
  std::vector<std::thread> pool;
  const uint64_t count = stop > start ? (stop - start + stride - 1) / stride : 0;
  for (int t = 0; t < threads; t++) {
    pool.emplace_back([&, t] {
      const uint64_t lo = count * t / threads, hi = count * (t + 1) / threads;
      for (uint64_t k = lo; k < hi; k++) {
        const uint32_t u = (uint32_t)(start + k * stride);
        float x;
        memcpy(&x, &u, 4);
        const float a = ref(which, x), b = mine(which, x);
        uint32_t ua, ub;
        memcpy(&ua, &a, 4);
        memcpy(&ub, &b, 4);
        if (ua != ub && !(isnan(a) && isnan(b))) {
          if (first[t] == UINT64_MAX) first[t] = u;
          bad[t]++;
        }
      }
    });
  }
  uint64_t total = 0;
  uint64_t f = UINT64_MAX;
  for (int t = 0; t < threads; t++) {
    pool[t].join();
    total += bad[t];
    if (first[t] < f) f = first[t];
  }
  if (first_bad) *first_bad = (uint32_t)(f == UINT64_MAX ? 0 : f);
  return total;
}

// ---- softplus and mish: the device's per-element rules (rt_ops.cuh) against
// the same formulas over this machine's glibc (the reference's libm) --------
static float act_ref(int which, float x) {
  const float sp = x > 20.0f ? x : logf(1.0f + expf(x));
  return which == 0 ? sp : x * tanhf(sp);
}

static float act_mine(int which, float x) {
  return which == 0 ? rt::OpSoftplus{}(x) : rt::OpMish{}(x);
}

static int64_t ordered(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  return u < 0x80000000u ? (int64_t)u : (int64_t)0x80000000u - (int64_t)u;
}

// Largest ulp distance between act_mine and act_ref over inputs u = start,
// start+stride, ... < stop (NaN inputs skipped; two NaN results are equal).
// *over receives how many inputs exceed `bound` ulp, *worst the input with
// the largest distance.
extern "C" uint64_t act_max_ulp(int which, uint64_t start, uint64_t stop, uint64_t stride,
                                int threads, uint64_t bound, uint64_t* over, uint32_t* worst) {
  if (threads < 1) threads = 1;
  std::vector<uint64_t> mx(threads, 0), cnt(threads, 0);
  std::vector<uint32_t> arg(threads, 0);
  std::vector<std::thread> pool;
  const uint64_t count = stop > start ? (stop - start + stride - 1) / stride : 0;
  for (int t = 0; t < threads; t++) {
    pool.emplace_back([&, t] {
      const uint64_t lo = count * t / threads, hi = count * (t + 1) / threads;
      for (uint64_t k = lo; k < hi; k++) {
        const uint32_t u = (uint32_t)(start + k * stride);
        float x;
        memcpy(&x, &u, 4);
        if (isnan(x)) continue;
        const float a = act_ref(which, x), b = act_mine(which, x);
        if (isnan(a) && isnan(b)) continue;
        const int64_t d = ordered(a) - ordered(b);
        const uint64_t ad = (uint64_t)(d < 0 ? -d : d);
        if (ad > bound) cnt[t]++;
        if (ad > mx[t]) {
          mx[t] = ad;
          arg[t] = u;
        }
      }
    });
  }
  uint64_t m = 0, c = 0;
  uint32_t w = 0;
  for (int t = 0; t < threads; t++) {
    pool[t].join();
    c += cnt[t];
    if (mx[t] > m) {
      m = mx[t];
      w = arg[t];
    }
  }
  if (over) *over = c;
  if (worst) *worst = w;
  return m;
}

// The device rule evaluated on the host (which: 0 softplus, 1 mish).
extern "C" void act_restated(int which, const float* x, float* out, uint64_t n) {
  for (uint64_t i = 0; i < n; i++) out[i] = act_mine(which, x[i]);
}

// Inputs u = start, start+stride, ... < stop where act_mine misses the
// north_star tolerance for transcendental activations against act_ref: more
// than 4 ulp AND more than 1e-6 relative error (NaN inputs skipped; two NaN
// results are equal).  *first receives the first such input.
extern "C" uint64_t act_tol_violations(int which, uint64_t start, uint64_t stop, uint64_t stride,
                                       int threads, uint32_t* first) {
  if (threads < 1) threads = 1;
  std::vector<uint64_t> cnt(threads, 0), fst(threads, UINT64_MAX);
  std::vector<std::thread> pool;
  const uint64_t count = stop > start ? (stop - start + stride - 1) / stride : 0;
  for (int t = 0; t < threads; t++) {
    pool.emplace_back([&, t] {
      const uint64_t lo = count * t / threads, hi = count * (t + 1) / threads;
      for (uint64_t k = lo; k < hi; k++) {
        const uint32_t u = (uint32_t)(start + k * stride);
        float x;
        memcpy(&x, &u, 4);
        if (isnan(x)) continue;
        const float a = act_ref(which, x), b = act_mine(which, x);
        if (isnan(a) && isnan(b)) continue;
        const int64_t d = ordered(a) - ordered(b);
        if ((d < 0 ? -d : d) <= 4) continue;
        const double rel = fabs((double)a - (double)b) / fabs((double)a);
        if (rel <= 1e-6) continue;
        if (fst[t] == UINT64_MAX) fst[t] = u;
        cnt[t]++;
      }
    });
  }
  uint64_t c = 0, f = UINT64_MAX;
  for (int t = 0; t < threads; t++) {
    pool[t].join();
    c += cnt[t];
    if (fst[t] < f) f = fst[t];
  }
  if (first) *first = (uint32_t)(f == UINT64_MAX ? 0 : f);
  return c;
}
