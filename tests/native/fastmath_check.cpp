// Host build of the tolerance math mode (rusttorch_b200/csrc/rt_fastmath.cuh
// and the *Tol rules of rt_ops.cuh), compared with the reference's formulas
// over this machine's glibc.  Every step of the device functions is one IEEE
// operation (or the correctly rounded reciprocal), so this build gives the
// device's bits; the GPU tests check that on a sweep of inputs.  Test
// infrastructure: built and loaded by tests/test_fastmath.py.
#include <math.h>
#include <stdint.h>
#include <string.h>

#include <thread>
#include <vector>

#include "../../rusttorch_b200/csrc/rt_ops.cuh"

namespace {

// sqrt(2/pi) in f32 as the reference computes it (activation.rs:69).
float gelu_k() { return sqrtf(2.0f / (float)M_PI); }

// The reference's per-element formulas over glibc (activation.rs), one
// rounding per f32 operation (built with -ffp-contract=off).
float ref(int which, float x) {
  switch (which) {
    case 0: return 1.0f / (1.0f + expf(-x));                           // sigmoid
    case 1: return x / (1.0f + expf(-x));                              // swish
    case 2: return tanhf(x);                                           // tanh
    case 3: return x > 20.0f ? x : logf(1.0f + expf(x));               // softplus
    case 4: {                                                          // mish
      const float sp = x > 20.0f ? x : logf(1.0f + expf(x));
      return x * tanhf(sp);
    }
    case 5: {                                                          // gelu
      const float inner = x + 0.044715f * ((x * x) * x);
      return (0.5f * x) * (1.0f + tanhf(gelu_k() * inner));
    }
    case 6: return expf(x);                                            // exp
    case 7: return x >= 1.17549435e-38f && x <= 3.40282347e38f ? logf(x) : NAN;  // log
    default: return NAN;
  }
}

float mine(int which, float x) {
  switch (which) {
    case 0: return rt::OpSigmoidTol{}(x);
    case 1: return rt::OpSwishTol{}(x);
    case 2: return rt::OpTanhTol{}(x);
    case 3: return rt::OpSoftplusTol{}(x);
    case 4: return rt::OpMishTol{}(x);
    case 5: return rt::OpGeluTol{gelu_k()}(x);
    case 6: return rt::exp_fast(x);
    case 7: {
      uint32_t u;
      memcpy(&u, &x, 4);
      // log_fast's domain: positive normal floats
      return (u >= 0x00800000u && u < 0x7f800000u) ? rt::log_fast(x) : NAN;
    }
    default: return NAN;
  }
}

int64_t ordered(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  return u < 0x80000000u ? (int64_t)u : (int64_t)0x80000000u - (int64_t)u;
}

}  // namespace

// The device rule evaluated on the host, for comparison with GPU results.
extern "C" void fm_eval(int which, const float* x, float* out, uint64_t n) {
  for (uint64_t i = 0; i < n; i++) out[i] = mine(which, x[i]);
}
extern "C" void fm_ref(int which, const float* x, float* out, uint64_t n) {
  for (uint64_t i = 0; i < n; i++) out[i] = ref(which, x[i]);
}

// Scan of inputs u = start, start+stride, ... < stop (NaN inputs skipped;
// two NaN results are equal, +0 and -0 are equal).  Returns the number of
// inputs that miss north_star's tolerance for transcendental activations
// (more than 4 ulp AND more than 1e-6 relative error); stats[0] = largest
// ulp distance, stats[1] = largest relative error over results that are
// normal floats, worst[0] = first violating input, worst[1] = the input with
// the largest ulp distance.
extern "C" uint64_t fm_scan(int which, uint64_t start, uint64_t stop, uint64_t stride,
                            int threads, double* stats, uint32_t* worst) {
  if (threads < 1) threads = 1;
  std::vector<uint64_t> cnt(threads, 0), fst(threads, UINT64_MAX), mxu(threads, 0);
  std::vector<uint32_t> arg(threads, 0);
  std::vector<double> mxr(threads, 0.0);
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
        const float a = ref(which, x), b = mine(which, x);
        if (isnan(a) && isnan(b)) continue;
        int64_t d = ordered(a) - ordered(b);
        if (isnan(a) != isnan(b)) d = INT64_MAX / 4;
        const uint64_t ad = (uint64_t)(d < 0 ? -d : d);
        if (ad > mxu[t]) {
          mxu[t] = ad;
          arg[t] = u;
        }
        double rel = 0.0;
        if (a != b) rel = fabs((double)a - (double)b) / fabs((double)a);
        if (isnan(rel) || isinf(rel)) rel = 1e300;
        if (fabsf(a) >= 1.17549435e-38f && rel > mxr[t]) mxr[t] = rel;
        if (ad <= 4 || rel <= 1e-6) continue;
        if (fst[t] == UINT64_MAX) fst[t] = u;
        cnt[t]++;
      }
    });
  }
  uint64_t c = 0, f = UINT64_MAX, m = 0;
  uint32_t w = 0;
  double r = 0.0;
  for (int t = 0; t < threads; t++) {
    pool[t].join();
    c += cnt[t];
    if (fst[t] < f) f = fst[t];
    if (mxu[t] > m) {
      m = mxu[t];
      w = arg[t];
    }
    if (mxr[t] > r) r = mxr[t];
  }
  if (stats) {
    stats[0] = (double)m;
    stats[1] = r;
  }
  if (worst) {
    worst[0] = (uint32_t)(f == UINT64_MAX ? 0 : f);
    worst[1] = w;
  }
  return c;
}

// Softmax along the last axis of a [rows, len] array as the device computes
// it in the tolerance mode: m = max (fmaxf), e = exp_fast_nonpos(x - m), s =
// ndarray's unrolled_fold of e (eight chains over i % 8 from 0.0, combined as
// 0 + (p0+p4) + (p1+p5) + (p2+p6) + (p3+p7), then the tail in order),
// y = e / s rounded once.
extern "C" void fm_softmax_rows(const float* x, uint64_t rows, uint64_t len, float* out,
                                int threads) {
  if (threads < 1) threads = 1;
  std::vector<std::thread> pool;
  for (int t = 0; t < threads; t++) {
    pool.emplace_back([=] {
      std::vector<float> e(len);
      for (uint64_t r = rows * t / threads; r < rows * (t + 1) / threads; r++) {
        const float* xr = x + r * len;
        float m = -INFINITY;
        for (uint64_t i = 0; i < len; i++) m = fmaxf(m, xr[i]);
        for (uint64_t i = 0; i < len; i++) e[i] = rt::exp_fast_nonpos(xr[i] - m);
        float p[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        const uint64_t steps = len / 8;
        for (uint64_t k = 0; k < steps; k++)
          for (int j = 0; j < 8; j++) p[j] = p[j] + e[8 * k + j];
        float acc = 0.0f;
        acc = acc + (p[0] + p[4]);
        acc = acc + (p[1] + p[5]);
        acc = acc + (p[2] + p[6]);
        acc = acc + (p[3] + p[7]);
        for (uint64_t i = steps * 8; i < len; i++) acc = acc + e[i];
        for (uint64_t i = 0; i < len; i++) out[r * len + i] = e[i] / acc;
      }
    });
  }
  for (auto& th : pool) th.join();
}
