// Host build of rusttorch_b200/csrc/rt_libm.cuh, compared with this
// machine's glibc (the reference's libm).  Test infrastructure: built and
// loaded by tests/test_libm_restatement.py.
#include <math.h>
#include <stdint.h>
#include <string.h>

#include <thread>
#include <vector>

#include "../../rusttorch_b200/csrc/rt_libm.cuh"

static float ref(int which, float x) {
  switch (which) {
    case 0: return expf(x);
    case 1: return expm1f(x);
    case 2: return tanhf(x);
    case 3: return logf(x);
    case 5: return expf(x);                  // 5: expf_glibc_nonpos (x <= 0, NaN)
    case 6: return (float)log((double)x);    // 6: logf_pos (positive normals, NaN)
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
