/*
 * rt_oracle.c — CPU restatement of rusttorch-core's hot path.
 *
 * TEST INFRASTRUCTURE ONLY (the parity checker; see rt_oracle.h).  Build with
 * oracle/Makefile: gcc -O2 -ffp-contract=off -fno-fast-math.
 */
#include "rt_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

/* ------------------------------------------------------------------------ */
/* threading (rayon stand-in for the ops the reference runs in parallel)    */
/* ------------------------------------------------------------------------ */

static int g_threads = 0;

void rto_set_threads(int n) { g_threads = n > 0 ? n : 0; }

int rto_get_threads(void) {
  if (g_threads > 0) return g_threads;
  long c = sysconf(_SC_NPROCESSORS_ONLN);
  return c > 0 ? (int)c : 1;
}

typedef struct {
  const float* a;
  const float* b;
  float* out;
  size_t lo, hi;
} add_job;

static void* add_worker(void* arg) {
  add_job* j = (add_job*)arg;
  for (size_t i = j->lo; i < j->hi; i++) j->out[i] = j->a[i] + j->b[i];
  return NULL;
}

/* core/src/ops/elementwise.rs:9 PARALLEL_THRESHOLD */
#define RT_PARALLEL_THRESHOLD 10000

/* core/src/ops/elementwise.rs:14-94: f32 add.  At n >= 10,000 the reference
 * clones `a` and runs `r += b` over rayon's pool (:31-43); the value of every
 * element is a[i] + b[i] either way. */
void rto_add(const float* a, const float* b, float* out, size_t n) {
  int t = rto_get_threads();
  if (n < RT_PARALLEL_THRESHOLD || t <= 1) {
    for (size_t i = 0; i < n; i++) out[i] = a[i] + b[i];
    return;
  }
  enum { MAXT = 256 };
  if (t > MAXT) t = MAXT;
  pthread_t th[MAXT];
  add_job jobs[MAXT];
  size_t chunk = (n + (size_t)t - 1) / (size_t)t;
  int started = 0;
  for (int k = 0; k < t; k++) {
    size_t lo = (size_t)k * chunk, hi = lo + chunk;
    if (lo >= n) break;
    if (hi > n) hi = n;
    jobs[k] = (add_job){a, b, out, lo, hi};
    if (pthread_create(&th[k], NULL, add_worker, &jobs[k]) != 0) {
      add_worker(&jobs[k]);
      th[k] = 0;
    }
    started++;
  }
  for (int k = 0; k < started; k++)
    if (th[k]) pthread_join(th[k], NULL);
}

/* core/src/ops/elementwise.rs:130-160 */
void rto_sub(const float* a, const float* b, float* out, size_t n) {
  for (size_t i = 0; i < n; i++) out[i] = a[i] - b[i];
}

/* core/src/ops/elementwise.rs:97-127 */
void rto_mul(const float* a, const float* b, float* out, size_t n) {
  for (size_t i = 0; i < n; i++) out[i] = a[i] * b[i];
}

/* core/src/ops/elementwise.rs:163-197 (IEEE division) */
void rto_div(const float* a, const float* b, float* out, size_t n) {
  for (size_t i = 0; i < n; i++) out[i] = a[i] / b[i];
}

/* core/src/ops/elementwise.rs:200-210 */
void rto_add_scalar(const float* x, float s, float* out, size_t n) {
  for (size_t i = 0; i < n; i++) out[i] = x[i] + s;
}

/* core/src/ops/elementwise.rs:213-223 */
void rto_mul_scalar(const float* x, float s, float* out, size_t n) {
  for (size_t i = 0; i < n; i++) out[i] = x[i] * s;
}

/* core/src/ops/simd.rs:275-370: a*b + c with two roundings (Rust never
 * contracts to an FMA; this file is compiled with -ffp-contract=off). */
void rto_fused_multiply_add(const float* a, const float* b, const float* c, float* out,
                            size_t n) {
  for (size_t i = 0; i < n; i++) {
    float p = a[i] * b[i];
    out[i] = p + c[i];
  }
}

/* ------------------------------------------------------------------------ */
/* activations                                                              */
/* ------------------------------------------------------------------------ */

/* core/src/ops/activation.rs:8-18: x.max(0.0).  f32::max is IEEE maxNum; on
 * x86_64 LLVM lowers maxnum(x, 0.0) with a never-NaN constant operand to
 * MAXSS(x, 0.0) = (x > 0 ? x : 0.0), so relu(NaN) = +0 and relu(-0) = +0. */
void rto_relu(const float* x, float* out, size_t n) {
  for (size_t i = 0; i < n; i++) out[i] = x[i] > 0.0f ? x[i] : 0.0f;
}

/* core/src/ops/activation.rs:170-191 */
void rto_leaky_relu(const float* x, float alpha, float* out, size_t n) {
  for (size_t i = 0; i < n; i++) out[i] = x[i] > 0.0f ? x[i] : alpha * x[i];
}

/* core/src/ops/activation.rs:21-37: 1.0 / (1.0 + (-x).exp()) */
void rto_sigmoid(const float* x, float* out, size_t n) {
  for (size_t i = 0; i < n; i++) {
    float e = expf(-x[i]);
    float d = 1.0f + e;
    out[i] = 1.0f / d;
  }
}

/* core/src/ops/activation.rs:40-56 */
void rto_tanh(const float* x, float* out, size_t n) {
  for (size_t i = 0; i < n; i++) out[i] = tanhf(x[i]);
}

/* sqrt_2_over_pi = (2.0_f32 / PI).sqrt(), core/src/ops/activation.rs:73 */
static float gelu_k(void) {
  volatile float two = 2.0f, pi = 3.14159265358979323846f; /* std::f32::consts::PI */
  float q = two / pi;
  return sqrtf(q);
}

/* core/src/ops/activation.rs:61-88:
 *   0.5 * x * (1.0 + (k * (x + 0.044715 * x.powi(3))).tanh())
 * `0.5 * x * (..)` associates as (0.5*x)*(..); powi(x,3) = (x*x)*x. */
void rto_gelu(const float* x, float* out, size_t n) {
  const float k = gelu_k();
  for (size_t i = 0; i < n; i++) {
    float v = x[i];
    float x2 = v * v;
    float x3 = x2 * v;
    float c = 0.044715f * x3;
    float inner = v + c;
    float z = k * inner;
    float t = tanhf(z);
    float h = 0.5f * v;
    float one_t = 1.0f + t;
    out[i] = h * one_t;
  }
}

/* core/src/ops/activation.rs:263-279: x / (1.0 + (-x).exp()) */
void rto_swish(const float* x, float* out, size_t n) {
  for (size_t i = 0; i < n; i++) {
    float e = expf(-x[i]);
    float d = 1.0f + e;
    out[i] = x[i] / d;
  }
}

/* core/src/ops/activation.rs:195-222; alpha <= 0 is rejected at :202-207. */
int rto_elu(const float* x, float alpha, float* out, size_t n) {
  if (alpha <= 0.0f) return RTO_INVALID_ARGUMENT;
  for (size_t i = 0; i < n; i++) {
    float v = x[i];
    if (v > 0.0f) {
      out[i] = v;
    } else {
      float em1 = expf(v) - 1.0f;
      out[i] = alpha * em1;
    }
  }
  return RTO_OK;
}

/* core/src/ops/activation.rs:228-259: f64 ALPHA/SCALE cast to f32 (:236-251) */
void rto_selu(const float* x, float* out, size_t n) {
  const double ALPHA = 1.6732632423543772;
  const double SCALE = 1.0507009873554805;
  const float a = (float)ALPHA, s = (float)SCALE;
  for (size_t i = 0; i < n; i++) {
    float v = x[i];
    float inner;
    if (v > 0.0f) {
      inner = v;
    } else {
      float em1 = expf(v) - 1.0f;
      inner = a * em1;
    }
    out[i] = s * inner;
  }
}

/* core/src/ops/activation.rs:319-346 */
static float softplus1(float v) {
  if (v > 20.0f) return v;
  float e = expf(v);
  float d = 1.0f + e;
  return logf(d);
}

/* core/src/ops/activation.rs:284-314: x * softplus(x).tanh() */
void rto_mish(const float* x, float* out, size_t n) {
  for (size_t i = 0; i < n; i++) {
    float sp = softplus1(x[i]);
    float t = tanhf(sp);
    out[i] = x[i] * t;
  }
}

void rto_softplus(const float* x, float* out, size_t n) {
  for (size_t i = 0; i < n; i++) out[i] = softplus1(x[i]);
}

/* core/src/ops/activation.rs:351-367: x / (1.0 + x.abs()) */
void rto_softsign(const float* x, float* out, size_t n) {
  for (size_t i = 0; i < n; i++) {
    float d = 1.0f + fabsf(x[i]);
    out[i] = x[i] / d;
  }
}

/* ------------------------------------------------------------------------ */
/* ordering helpers (Rust core::cmp)                                        */
/* ------------------------------------------------------------------------ */

/* Iterator::max_by(|a,b| a.partial_cmp(b).unwrap_or(Equal)) folds with
 * cmp::max_by(acc, x): Greater -> acc, Less|Equal -> x.  Unordered (NaN)
 * compares Equal, so: acc = (acc > x) ? acc : x. */
static inline float max2(float acc, float x) { return acc > x ? acc : x; }
/* cmp::min_by(acc, x): Less|Equal -> acc, Greater -> x. */
static inline float min2(float acc, float x) { return acc > x ? x : acc; }

/* ndarray 0.15 numeric_util::unrolled_fold(xs, zero, add) over a strided lane:
 * eight partial sums p0..p7 over consecutive groups of 8, combined as
 * acc = 0 + (p0+p4); acc += (p1+p5); acc += (p2+p6); acc += (p3+p7), then the
 * (< 8) remaining elements are added in order. */
static float unrolled_sum(const float* x, size_t len, size_t stride) {
  float p[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  size_t i = 0;
  for (; i + 8 <= len; i += 8)
    for (int j = 0; j < 8; j++) p[j] = p[j] + x[(i + (size_t)j) * stride];
  float acc = 0.0f;
  acc = acc + (p[0] + p[4]);
  acc = acc + (p[1] + p[5]);
  acc = acc + (p[2] + p[6]);
  acc = acc + (p[3] + p[7]);
  for (; i < len; i++) acc = acc + x[i * stride];
  return acc;
}

float rto_unrolled_sum_f32(const float* x, size_t n) { return unrolled_sum(x, n, 1); }

/* Iterator::sum::<f32>() over x: init + x[0] + x[1] + ... (init = -0.0 in the
 * reference; core's Sum for f32 folds from -0.0). */
float rto_chain_sum_f32(const float* x, size_t n, float init) {
  float acc = init;
  for (size_t i = 0; i < n; i++) acc = acc + x[i];
  return acc;
}

static void split_dims(const size_t* shape, size_t ndim, size_t dim, size_t* outer, size_t* len,
                       size_t* inner) {
  size_t o = 1, in = 1;
  for (size_t d = 0; d < dim; d++) o *= shape[d];
  for (size_t d = dim + 1; d < ndim; d++) in *= shape[d];
  *outer = o;
  *len = shape[dim];
  *inner = in;
}

/* ndarray 0.15 ArrayBase::sum_axis(Axis(dim)) on a C-contiguous f32 array:
 * if dim is the minimum-stride axis (always the last axis of a C-contiguous
 * array) every lane is reduced with unrolled_fold; otherwise
 * `res = zeros; for sub in axis_iter(dim) { res = res + &sub }`, i.e. each
 * output element is ((0 + x_0) + x_1) + ... in index order along dim. */
static void sum_axis(const float* x, const size_t* shape, size_t ndim, size_t dim, float* out) {
  size_t outer, len, inner;
  split_dims(shape, ndim, dim, &outer, &len, &inner);
  if (dim == ndim - 1) {
    for (size_t o = 0; o < outer; o++) out[o] = unrolled_sum(x + o * len, len, 1);
    return;
  }
  for (size_t o = 0; o < outer; o++) {
    float* r = out + o * inner;
    for (size_t i = 0; i < inner; i++) r[i] = 0.0f;
    for (size_t l = 0; l < len; l++) {
      const float* row = x + (o * len + l) * inner;
      for (size_t i = 0; i < inner; i++) r[i] = r[i] + row[i];
    }
  }
}

/* core/src/ops/activation.rs:92-167 (f32 arm :109-137):
 *   m = map_axis(dim, max_by fold).unwrap_or(0.0)
 *   e = (x - m).exp()
 *   s = e.sum_axis(dim)          (ndarray order, see sum_axis)
 *   y = e / s                                                              */
int rto_softmax(const float* x, const size_t* shape, size_t ndim, size_t dim, float* out) {
  if (dim >= ndim) return RTO_INVALID_DIMENSION;
  size_t outer, len, inner;
  split_dims(shape, ndim, dim, &outer, &len, &inner);
  size_t lanes = outer * inner;
  if (lanes == 0 || len == 0) return RTO_OK;
  /* scratch for m and s, one per lane */
  float* m = (float*)malloc(lanes * sizeof(float));
  float* s = (float*)malloc(lanes * sizeof(float));
  if (!m || !s) {
    free(m);
    free(s);
    return RTO_INVALID_ARGUMENT;
  }
  for (size_t o = 0; o < outer; o++)
    for (size_t i = 0; i < inner; i++) {
      const float* lane = x + o * len * inner + i;
      float acc = lane[0];
      for (size_t l = 1; l < len; l++) acc = max2(acc, lane[l * inner]);
      m[o * inner + i] = acc;
    }
  for (size_t o = 0; o < outer; o++)
    for (size_t l = 0; l < len; l++)
      for (size_t i = 0; i < inner; i++) {
        size_t k = (o * len + l) * inner + i;
        float d = x[k] - m[o * inner + i];
        out[k] = expf(d);
      }
  sum_axis(out, shape, ndim, dim, s);
  for (size_t o = 0; o < outer; o++)
    for (size_t l = 0; l < len; l++)
      for (size_t i = 0; i < inner; i++) {
        size_t k = (o * len + l) * inner + i;
        out[k] = out[k] / s[o * inner + i];
      }
  free(m);
  free(s);
  return RTO_OK;
}

/* ------------------------------------------------------------------------ */
/* reductions                                                               */
/* ------------------------------------------------------------------------ */

/* core/src/ops/reduction.rs:7-14: arr.iter().map(|&x| x as f64).sum() —
 * one sequential f64 fold in index order. */
double rto_sum(const float* x, size_t n) {
  double acc = 0.0;
  for (size_t i = 0; i < n; i++) acc = acc + (double)x[i];
  return acc;
}

/* core/src/ops/reduction.rs:17-26 */
int rto_mean(const float* x, size_t n, double* out) {
  if (n == 0) return RTO_EMPTY_TENSOR;
  *out = rto_sum(x, n) / (double)n;
  return RTO_OK;
}

/* core/src/ops/reduction.rs:29-49 */
int rto_max(const float* x, size_t n, double* out) {
  if (n == 0) return RTO_EMPTY_TENSOR;
  float acc = x[0];
  for (size_t i = 1; i < n; i++) acc = max2(acc, x[i]);
  *out = (double)acc;
  return RTO_OK;
}

/* core/src/ops/reduction.rs:52-72 */
int rto_min(const float* x, size_t n, double* out) {
  if (n == 0) return RTO_EMPTY_TENSOR;
  float acc = x[0];
  for (size_t i = 1; i < n; i++) acc = min2(acc, x[i]);
  *out = (double)acc;
  return RTO_OK;
}

/* core/src/ops/reduction.rs:75-108 (f32 arm :86-91) */
int rto_sum_dim(const float* x, const size_t* shape, size_t ndim, size_t dim, float* out) {
  if (dim >= ndim) return RTO_INVALID_DIMENSION;
  sum_axis(x, shape, ndim, dim, out);
  return RTO_OK;
}

/* core/src/ops/reduction.rs:111-150 (f32 arm :121-127): ndarray mean_axis =
 * sum_axis(dim) / (len as f32).  A zero-length axis makes mean_axis return
 * None and the reference unwrap() panic; the oracle reports EmptyTensor. */
int rto_mean_dim(const float* x, const size_t* shape, size_t ndim, size_t dim, float* out) {
  if (dim >= ndim) return RTO_INVALID_DIMENSION;
  size_t outer, len, inner;
  split_dims(shape, ndim, dim, &outer, &len, &inner);
  if (len == 0) return RTO_EMPTY_TENSOR;
  sum_axis(x, shape, ndim, dim, out);
  const float flen = (float)len;
  for (size_t k = 0; k < outer * inner; k++) out[k] = out[k] / flen;
  return RTO_OK;
}

/* Max along a dim (new op: the reference has none).  Each lane is folded
 * exactly like core/src/ops/reduction.rs:36-40. */
int rto_max_dim(const float* x, const size_t* shape, size_t ndim, size_t dim, float* out) {
  if (dim >= ndim) return RTO_INVALID_DIMENSION;
  size_t outer, len, inner;
  split_dims(shape, ndim, dim, &outer, &len, &inner);
  if (len == 0) return RTO_EMPTY_TENSOR;
  for (size_t o = 0; o < outer; o++)
    for (size_t i = 0; i < inner; i++) {
      const float* lane = x + o * len * inner + i;
      float acc = lane[0];
      for (size_t l = 1; l < len; l++) acc = max2(acc, lane[l * inner]);
      out[o * inner + i] = acc;
    }
  return RTO_OK;
}

/* ------------------------------------------------------------------------ */
/* optimizer update rules                                                   */
/* ------------------------------------------------------------------------ */

/* core/src/ops/optimizer.rs:242-271: the hyperparameter checks, in order.
 * NaN passes every check (the comparisons are false), as in the reference. */
static int adam_checks(double lr, double b1, double b2, double eps, uint64_t t) {
  if (lr <= 0.0) return RTO_INVALID_ARGUMENT;
  if (b1 <= 0.0 || b1 >= 1.0) return RTO_INVALID_ARGUMENT;
  if (b2 <= 0.0 || b2 >= 1.0) return RTO_INVALID_ARGUMENT;
  if (eps <= 0.0) return RTO_INVALID_ARGUMENT;
  if (t == 0) return RTO_INVALID_ARGUMENT;
  return RTO_OK;
}

/* core/src/ops/optimizer.rs:207-354 (f32 arm :284-315).  Bias corrections
 * in f64 with powf (:278-282), every other step in f32:
 *   m' = m*b1 + g*(1-b1);  v' = v*b2 + (g*g)*(1-b2)
 *   mh = m'/bc1; vh = v'/bc2; den = sqrt(vh) + eps; p' = p - (mh/den)*lr   */
int rto_adam_update(const float* p, const float* g, const float* m, const float* v, size_t n,
                    double lr, double beta1, double beta2, double eps, uint64_t t,
                    float* p_out, float* m_out, float* v_out) {
  int rc = adam_checks(lr, beta1, beta2, eps, t);
  if (rc) return rc;
  const double td = (double)t;
  const double bc1 = 1.0 - pow(beta1, td);
  const double bc2 = 1.0 - pow(beta2, td);
  const float b1 = (float)beta1, b2 = (float)beta2;
  const float omb1 = 1.0f - b1, omb2 = 1.0f - b2;
  const float fbc1 = (float)bc1, fbc2 = (float)bc2, feps = (float)eps, flr = (float)lr;
  for (size_t i = 0; i < n; i++) {
    float gi = g[i];
    float nm = m[i] * b1;
    float gm = gi * omb1;
    nm = nm + gm;
    float g2 = gi * gi;
    float nv = v[i] * b2;
    float gv = g2 * omb2;
    nv = nv + gv;
    float mh = nm / fbc1;
    float vh = nv / fbc2;
    float den = sqrtf(vh) + feps;
    float upd = mh / den;
    float step = upd * flr;
    float np = p[i] - step;
    p_out[i] = np;
    m_out[i] = nm;
    v_out[i] = nv;
  }
  return RTO_OK;
}

/* core/src/ops/optimizer.rs:379-440: weight_decay < 0 rejected first
 * (:392-397); Adam as above; then, if wd > 0, p'' = p' - p*(f32)(lr*wd)
 * with lr*wd computed in f64 (:413-421). */
int rto_adamw_update(const float* p, const float* g, const float* m, const float* v, size_t n,
                     double lr, double beta1, double beta2, double eps, double weight_decay,
                     uint64_t t, float* p_out, float* m_out, float* v_out) {
  if (weight_decay < 0.0) return RTO_INVALID_ARGUMENT;
  int rc = adam_checks(lr, beta1, beta2, eps, t);
  if (rc) return rc;
  if (!(weight_decay > 0.0))
    return rto_adam_update(p, g, m, v, n, lr, beta1, beta2, eps, t, p_out, m_out, v_out);
  const float lrwd = (float)(lr * weight_decay);
  const double td = (double)t;
  const double bc1 = 1.0 - pow(beta1, td);
  const double bc2 = 1.0 - pow(beta2, td);
  const float b1 = (float)beta1, b2 = (float)beta2;
  const float omb1 = 1.0f - b1, omb2 = 1.0f - b2;
  const float fbc1 = (float)bc1, fbc2 = (float)bc2, feps = (float)eps, flr = (float)lr;
  for (size_t i = 0; i < n; i++) {
    float pi = p[i], gi = g[i];
    float nm = m[i] * b1;
    float gm = gi * omb1;
    nm = nm + gm;
    float g2 = gi * gi;
    float nv = v[i] * b2;
    float gv = g2 * omb2;
    nv = nv + gv;
    float mh = nm / fbc1;
    float vh = nv / fbc2;
    float den = sqrtf(vh) + feps;
    float upd = mh / den;
    float step = upd * flr;
    float pa = pi - step;
    float decay = pi * lrwd;
    p_out[i] = pa - decay;
    m_out[i] = nm;
    v_out[i] = nv;
  }
  return RTO_OK;
}

/* core/src/ops/optimizer.rs:42-86 (f32 arm :72-74): p - g*(f32)lr */
int rto_sgd_update(const float* p, const float* g, size_t n, double lr, float* p_out) {
  if (lr <= 0.0) return RTO_INVALID_ARGUMENT;
  const float flr = (float)lr;
  for (size_t i = 0; i < n; i++) {
    float step = g[i] * flr;
    p_out[i] = p[i] - step;
  }
  return RTO_OK;
}

/* core/src/ops/optimizer.rs:108-177 (f32 arm :150-153):
 *   v' = v*(f32)mom + g;  p' = p - v'*(f32)lr;  momentum must be in [0,1) */
int rto_sgd_momentum_update(const float* p, const float* g, const float* vel, size_t n,
                            double lr, double momentum, float* p_out, float* vel_out) {
  if (lr <= 0.0) return RTO_INVALID_ARGUMENT;
  if (!(momentum >= 0.0 && momentum < 1.0)) return RTO_INVALID_ARGUMENT;
  const float fm = (float)momentum, flr = (float)lr;
  for (size_t i = 0; i < n; i++) {
    float nv = vel[i] * fm;
    nv = nv + g[i];
    float step = nv * flr;
    p_out[i] = p[i] - step;
    vel_out[i] = nv;
  }
  return RTO_OK;
}

/* ------------------------------------------------------------------------ */
/* nn optimizers (core/src/nn/optim.rs)                                     */
/* ------------------------------------------------------------------------ */

/* Adam::step, nn/optim.rs:262-313: bias corrections in f32 with powf
 * (:266-268), then per element (:297-304)
 *   m' = b1*m + (1-b1)*g;  v' = b2*v + ((1-b2)*g)*g
 *   p' = p - (lr*(m'/bc1)) / (sqrt(v'/bc2) + eps)                          */
void rto_nn_adam_step(const float* p, const float* g, const float* m, const float* v, size_t n,
                      float lr, float beta1, float beta2, float eps, uint64_t t, float* p_out,
                      float* m_out, float* v_out) {
  const float tf = (float)t;
  const float bc1 = 1.0f - powf(beta1, tf);
  const float bc2 = 1.0f - powf(beta2, tf);
  const float omb1 = 1.0f - beta1, omb2 = 1.0f - beta2;
  for (size_t j = 0; j < n; j++) {
    float a = beta1 * m[j];
    float b = omb1 * g[j];
    float nm = a + b;
    float c = beta2 * v[j];
    float d = omb2 * g[j];
    d = d * g[j];
    float nv = c + d;
    float mh = nm / bc1;
    float vh = nv / bc2;
    float num = lr * mh;
    float den = sqrtf(vh) + eps;
    float q = num / den;
    p_out[j] = p[j] - q;
    m_out[j] = nm;
    v_out[j] = nv;
  }
}

/* SGD::step, nn/optim.rs:168-203:
 *   momentum > 0: v' = (momentum*v + g) + wd*p;  p' = p - lr*v'
 *   otherwise:    p' = p - lr*(g + wd*p)                                    */
void rto_nn_sgd_step(const float* p, const float* g, const float* vel, size_t n, float lr,
                     float momentum, float weight_decay, float* p_out, float* vel_out) {
  for (size_t j = 0; j < n; j++) {
    if (momentum > 0.0f) {
      float a = momentum * vel[j];
      a = a + g[j];
      float b = weight_decay * p[j];
      float nv = a + b;
      float step = lr * nv;
      vel_out[j] = nv;
      p_out[j] = p[j] - step;
    } else {
      float b = weight_decay * p[j];
      float e = g[j] + b;
      float step = lr * e;
      p_out[j] = p[j] - step;
    }
  }
}

/* ------------------------------------------------------------------------ */
/* loss functions (core/src/ops/loss.rs)                                    */
/* ------------------------------------------------------------------------ */

/* ndarray's arithmetic allocates each intermediate (diff, squared, ...) and
 * sum() folds the last one with unrolled_fold; the terms are computed here
 * into one buffer first, in the same f32 operations. */
static double terms_mean8(float* terms, size_t n) {
  const float s = unrolled_sum(terms, n, 1);
  free(terms);
  return (double)s / (double)n;
}

double rto_mse_loss(const float* p, const float* t, size_t n) {
  float* d = (float*)malloc((n ? n : 1) * sizeof(float));
  for (size_t i = 0; i < n; i++) {
    float diff = p[i] - t[i]; /* :72 pred - targ */
    d[i] = diff * diff;       /* :73 &diff * &diff; :74 sum() */
  }
  return terms_mean8(d, n);
}

double rto_l1_loss(const float* p, const float* t, size_t n) {
  float* d = (float*)malloc((n ? n : 1) * sizeof(float));
  for (size_t i = 0; i < n; i++) d[i] = fabsf(p[i] - t[i]); /* :133-134 */
  return terms_mean8(d, n);
}

/* :204-213: |x| < beta ? 0.5*x*x/beta : |x| - 0.5*beta, beta as f32 */
double rto_smooth_l1_loss(const float* p, const float* t, size_t n, double beta) {
  const float b = (float)beta;
  float* d = (float*)malloc((n ? n : 1) * sizeof(float));
  for (size_t i = 0; i < n; i++) {
    float x = p[i] - t[i];
    float ax = fabsf(x);
    if (ax < b) {
      float h = 0.5f * x;
      h = h * x;
      d[i] = h / b;
    } else {
      float hb = 0.5f * b;
      d[i] = ax - hb;
    }
  }
  return terms_mean8(d, n);
}

/* f32::max / f32::min: the other operand when one is NaN (IEEE maxNum). */
static float rust_max(float a, float b) { return a != a ? b : (b != b ? a : (a > b ? a : b)); }
static float rust_min(float a, float b) { return a != a ? b : (b != b ? a : (a < b ? a : b)); }

/* :284-292: the terms folded in order by Iterator::sum::<f32>() (from -0.0) */
double rto_bce_loss(const float* p, const float* t, size_t n, double epsilon) {
  const float e = (float)epsilon;
  const float hi = 1.0f - e;
  float acc = -0.0f;
  for (size_t i = 0; i < n; i++) {
    float pc = rust_min(rust_max(p[i], e), hi);
    float a = t[i] * logf(pc);
    float om = 1.0f - t[i];
    float b = om * logf(1.0f - pc);
    float s = a + b;
    acc = acc + (-s);
  }
  return (double)acc / (double)n;
}

/* :363-370: -t * ln(max(p, eps)), folded in order from -0.0 */
double rto_ce_loss(const float* p, const float* t, size_t n, double epsilon) {
  const float e = (float)epsilon;
  float acc = -0.0f;
  for (size_t i = 0; i < n; i++) {
    float pc = rust_max(p[i], e);
    float term = (-t[i]) * logf(pc);
    acc = acc + term;
  }
  return (double)acc / (double)n;
}

/* ------------------------------------------------------------------------ */
/* autograd backward (core/src/autograd/ops.rs)                             */
/* ------------------------------------------------------------------------ */

/* :380-387: mask = x > 0 ? 1 : 0, then ops::mul(grad_output, mask) */
void rto_relu_backward(const float* g, const float* x, float* out, size_t n) {
  for (size_t i = 0; i < n; i++) {
    float mask = x[i] > 0.0f ? 1.0f : 0.0f;
    out[i] = g[i] * mask;
  }
}

/* :424-427: one_minus = sub(ones, y); sig_grad = mul(y, one_minus);
 * grad = mul(grad_output, sig_grad) */
void rto_sigmoid_backward(const float* g, const float* y, float* out, size_t n) {
  for (size_t i = 0; i < n; i++) {
    float one_minus = 1.0f - y[i];
    float sig_grad = y[i] * one_minus;
    out[i] = g[i] * sig_grad;
  }
}

/* :465-468: sq = mul(y, y); one_minus = sub(ones, sq); grad = mul(g, one_minus) */
void rto_tanh_backward(const float* g, const float* y, float* out, size_t n) {
  for (size_t i = 0; i < n; i++) {
    float sq = y[i] * y[i];
    float one_minus = 1.0f - sq;
    out[i] = g[i] * one_minus;
  }
}

static float sqrt_2_over_pi(void) {
  volatile float two = 2.0f, pi = 3.14159265358979323846f;
  return sqrtf(two / pi);
}

/* :3108-3118, each Rust f32 expression left to right */
void rto_gelu_backward(const float* g, const float* x, float* out, size_t n) {
  const float k = sqrt_2_over_pi();
  volatile float three = 3.0f, c = 0.044715f;
  const float c3 = three * c; /* `3.0 * 0.044715` in f32 */
  for (size_t i = 0; i < n; i++) {
    float xi = x[i];
    float x3 = xi * xi;
    x3 = x3 * xi;
    float t0 = 0.044715f * x3;
    t0 = xi + t0;
    float inner = k * t0;
    float t = tanhf(inner);
    float tt = t * t;
    float sech2 = 1.0f - tt;
    float d = c3 * xi;
    d = d * xi;
    d = 1.0f + d;
    float d_inner = k * d;
    float a = 1.0f + t;
    a = 0.5f * a;
    float b = 0.5f * xi;
    b = b * sech2;
    b = b * d_inner;
    float s = a + b;
    out[i] = g[i] * s;
  }
}

/* :3136-3141: 0.5 * x * (1.0 + (k * (x + 0.044715 * x * x * x)).tanh()) */
void rto_autograd_gelu(const float* x, float* out, size_t n) {
  const float k = sqrt_2_over_pi();
  for (size_t i = 0; i < n; i++) {
    float xi = x[i];
    float c = 0.044715f * xi;
    c = c * xi;
    c = c * xi;
    float inner = xi + c;
    inner = k * inner;
    float t = tanhf(inner);
    float h = 0.5f * xi;
    float one_t = 1.0f + t;
    out[i] = h * one_t;
  }
}

/* :179-188: grad_output.clone() and grad_output.neg() (a sign flip) */
void rto_sub_backward(const float* g, float* ga, float* gb, size_t n) {
  for (size_t i = 0; i < n; i++) {
    if (ga) ga[i] = g[i];
    if (gb) gb[i] = -g[i];
  }
}

/* :222-231: mul(g, b) and mul(g, a) */
void rto_mul_backward(const float* g, const float* a, const float* b, float* ga, float* gb,
                      size_t n) {
  for (size_t i = 0; i < n; i++) {
    if (ga) ga[i] = g[i] * b[i];
    if (gb) gb[i] = g[i] * a[i];
  }
}

/* :271-289: div(g, b); b_sq = mul(b, b); neg_a = a.neg();
 * q = div(neg_a, b_sq); mul(g, q) */
void rto_div_backward(const float* g, const float* a, const float* b, float* ga, float* gb,
                      size_t n) {
  for (size_t i = 0; i < n; i++) {
    if (ga) ga[i] = g[i] / b[i];
    if (gb) {
      float b_sq = b[i] * b[i];
      float neg_a = -a[i];
      float q = neg_a / b_sq;
      gb[i] = g[i] * q;
    }
  }
}

void rto_fill_backward(float g, float* out, size_t n, int mean) {
  const float v = mean ? (float)((double)g / (double)n) : (float)(double)g;
  for (size_t i = 0; i < n; i++) out[i] = v;
}

static size_t numel_of(const size_t* s, size_t nd) {
  size_t t = 1;
  for (size_t i = 0; i < nd; i++) t *= s[i];
  return t;
}

/* reduce_to_shape, :627-681, branch for branch */
int rto_reduce_to_shape(const float* grad, const size_t* gshape, size_t gnd, float* out,
                        const size_t* oshape, size_t ond) {
  const size_t len = numel_of(gshape, gnd), m = numel_of(oshape, ond);
  int same = gnd == ond;
  for (size_t i = 0; same && i < gnd; i++) same = gshape[i] == oshape[i];
  if (same) {
    memcpy(out, grad, len * sizeof(float));
    return RTO_OK;
  }
  if (gnd == 2 && ond == 2) {
    const size_t R = gshape[0], C = gshape[1];
    if (oshape[0] == 1 && oshape[1] == C) {
      for (size_t c = 0; c < C; c++) out[c] = 0.0f;
      for (size_t r = 0; r < R; r++)
        for (size_t c = 0; c < C; c++) out[c] += grad[r * C + c];
      return RTO_OK;
    }
    if (oshape[1] == 1 && oshape[0] == R) {
      for (size_t r = 0; r < R; r++) out[r] = 0.0f;
      for (size_t r = 0; r < R; r++)
        for (size_t c = 0; c < C; c++) out[r] += grad[r * C + c];
      return RTO_OK;
    }
  }
  if (len == m) {
    memcpy(out, grad, len * sizeof(float));
    return RTO_OK;
  }
  if (m == 0) return RTO_INVALID_ARGUMENT;
  for (size_t j = 0; j < m; j++) out[j] = 0.0f;
  for (size_t i = 0; i < len; i++) out[i % m] += grad[i];
  return RTO_OK;
}

/* ------------------------------------------------------------------------ */
/* broadcasting (core/src/ops/broadcast.rs)                                 */
/* ------------------------------------------------------------------------ */

/* broadcast_shape (:32-53) then the elementwise op on the materialised
 * copies (:177-198): element i of the result combines the elements of a and
 * b at i's coordinates, size-1 (or missing leading) dims repeating. */
int rto_broadcast_binary(int op, const float* a, const size_t* ashape, size_t andim,
                         const float* b, const size_t* bshape, size_t bndim, float* out) {
  enum { MAXD = 16 };
  size_t nd = andim > bndim ? andim : bndim;
  if (nd > MAXD) return RTO_INVALID_ARGUMENT;
  size_t oshape[MAXD], as[MAXD], bs[MAXD];
  for (size_t i = 0; i < nd; i++) {
    size_t da = i < nd - andim ? 1 : ashape[i - (nd - andim)];
    size_t db = i < nd - bndim ? 1 : bshape[i - (nd - bndim)];
    if (da != db && da != 1 && db != 1) return RTO_BROADCAST_ERROR;
    oshape[i] = da > db ? da : db;
    as[i] = da;
    bs[i] = db;
  }
  size_t total = 1;
  for (size_t i = 0; i < nd; i++) total *= oshape[i];
  for (size_t idx = 0; idx < total; idx++) {
    size_t rem = idx, ao = 0, bo = 0, am = 1, bm = 1;
    for (size_t k = nd; k-- > 0;) {
      size_t c = rem % oshape[k];
      rem /= oshape[k];
      ao += (as[k] == 1 ? 0 : c) * am;
      bo += (bs[k] == 1 ? 0 : c) * bm;
      am *= as[k];
      bm *= bs[k];
    }
    float x = a[ao], y = b[bo];
    switch (op) {
      case 0: out[idx] = x + y; break;
      case 1: out[idx] = x - y; break;
      case 2: out[idx] = x * y; break;
      default: out[idx] = x / y; break;
    }
  }
  return RTO_OK;
}

/* ------------------------------------------------------------------------ */
/* seeded generator                                                         */
/* ------------------------------------------------------------------------ */

static inline uint64_t splitmix64_at(uint64_t seed, uint64_t i) {
  uint64_t z = seed + (i + 1) * 0x9E3779B97F4A7C15ULL;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
  return z ^ (z >> 31);
}

typedef struct {
  float* out;
  size_t lo, hi;
  uint64_t seed, offset;
  float a, b;
  int normal;
} fill_job;

static void* fill_worker(void* arg) {
  fill_job* j = (fill_job*)arg;
  if (!j->normal) {
    const double span = (double)j->b - (double)j->a;
    for (size_t i = j->lo; i < j->hi; i++) {
      uint64_t z = splitmix64_at(j->seed, j->offset + i);
      double u = (double)(z >> 40) * 0x1p-24;
      j->out[i] = (float)((double)j->a + span * u);
    }
  } else {
    const double two_pi = 6.283185307179586;
    for (size_t i = j->lo; i < j->hi; i++) {
      uint64_t z = splitmix64_at(j->seed, j->offset + i);
      double u1 = ((double)(z >> 38) + 0.5) * 0x1p-26;
      double u2 = (double)((z >> 12) & 0x3FFFFFFULL) * 0x1p-26;
      double r = sqrt(-2.0 * log(u1)) * cos(two_pi * u2);
      j->out[i] = (float)((double)j->a + (double)j->b * r);
    }
  }
  return NULL;
}

/* Element i depends only on (seed, offset + i), so the split over threads
 * does not change any value. */
static void fill(float* out, size_t n, uint64_t seed, uint64_t offset, float a, float b,
                 int normal) {
  int t = rto_get_threads();
  enum { MAXT = 256 };
  if (t > MAXT) t = MAXT;
  if (n < (1u << 16)) t = 1;
  pthread_t th[MAXT];
  fill_job jobs[MAXT];
  size_t chunk = (n + (size_t)t - 1) / (size_t)t;
  int started = 0;
  for (int k = 0; k < t; k++) {
    size_t lo = (size_t)k * chunk, hi = lo + chunk;
    if (lo >= n) break;
    if (hi > n) hi = n;
    jobs[k] = (fill_job){out, lo, hi, seed, offset, a, b, normal};
    if (t == 1 || pthread_create(&th[k], NULL, fill_worker, &jobs[k]) != 0) {
      fill_worker(&jobs[k]);
      th[k] = 0;
    }
    started++;
  }
  for (int k = 0; k < started; k++)
    if (th[k]) pthread_join(th[k], NULL);
}

void rto_fill_uniform(float* out, size_t n, uint64_t seed, uint64_t offset, float lo, float hi) {
  fill(out, n, seed, offset, lo, hi, 0);
}

void rto_fill_normal(float* out, size_t n, uint64_t seed, uint64_t offset, float mean, float std) {
  fill(out, n, seed, offset, mean, std, 1);
}
