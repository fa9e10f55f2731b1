/*
 * rt_oracle.h — CPU restatement of rusttorch-core's data-parallel hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker for the CUDA
 * path in rusttorch_b200/.  Only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / reference leg of bench.py may load it.  The product never
 * links, calls or falls back to it.
 *
 * Every function restates one reference function, in the reference's f32
 * operation order, and cites the file:line it follows (paths relative to the
 * rusttorch repository root; "core/" = rusttorch-core/).  Compile with
 * -ffp-contract=off -fno-fast-math so that each f32 operation rounds once, as
 * Rust (which never contracts a*b+c) does.  Transcendentals call glibc libm
 * (expf/tanhf/logf), which is what Rust's f32::exp/tanh/ln lower to on
 * x86_64-linux-gnu.
 *
 * Third-party arithmetic the reference delegates to, restated here:
 *  - ndarray 0.15 (rusttorch Cargo.toml:15; no Cargo.lock, so 0.15.x is not
 *    pinned further): ArrayBase::sum_axis / mean_axis (order of the dim sums
 *    and of softmax's row sum) and numeric_util::unrolled_fold (eight-way
 *    unrolled lane sum).  No reference test checks these values, so this part
 *    of the oracle is pinned only by the restatement itself.
 *  - Rust core: Iterator::max_by/min_by via cmp::max_by/min_by (ties and NaN
 *    ordering of max/min), f32::max (relu), f64::powf (glibc pow).
 *
 * Error codes mirror core/src/error.rs:10-67 (see RTO_* below) and are the
 * same numbers the CUDA C-ABI returns.
 */
#ifndef RT_ORACLE_H
#define RT_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  RTO_OK = 0,
  RTO_SHAPE_MISMATCH = 1,
  RTO_DTYPE_MISMATCH = 2,
  RTO_EMPTY_TENSOR = 3,
  RTO_INVALID_DIMENSION = 4,
  RTO_INVALID_ARGUMENT = 5,
  RTO_BROADCAST_ERROR = 9,
};

/* ---- elementwise: core/src/ops/elementwise.rs, core/src/ops/simd.rs ---- */
void rto_add(const float* a, const float* b, float* out, size_t n);
void rto_sub(const float* a, const float* b, float* out, size_t n);
void rto_mul(const float* a, const float* b, float* out, size_t n);
void rto_div(const float* a, const float* b, float* out, size_t n);
void rto_add_scalar(const float* x, float s, float* out, size_t n);
void rto_mul_scalar(const float* x, float s, float* out, size_t n);
void rto_fused_multiply_add(const float* a, const float* b, const float* c, float* out, size_t n);

/* ---- activations: core/src/ops/activation.rs ---- */
void rto_relu(const float* x, float* out, size_t n);
void rto_leaky_relu(const float* x, float alpha, float* out, size_t n);
void rto_sigmoid(const float* x, float* out, size_t n);
void rto_tanh(const float* x, float* out, size_t n);
void rto_gelu(const float* x, float* out, size_t n);
void rto_swish(const float* x, float* out, size_t n);
int  rto_elu(const float* x, float alpha, float* out, size_t n);
void rto_selu(const float* x, float* out, size_t n);
void rto_mish(const float* x, float* out, size_t n);
void rto_softplus(const float* x, float* out, size_t n);
void rto_softsign(const float* x, float* out, size_t n);
/* softmax along `dim` of a C-contiguous tensor. */
int  rto_softmax(const float* x, const size_t* shape, size_t ndim, size_t dim, float* out);

/* ---- reductions: core/src/ops/reduction.rs ---- */
double rto_sum(const float* x, size_t n);
int    rto_mean(const float* x, size_t n, double* out);
int    rto_max(const float* x, size_t n, double* out);
int    rto_min(const float* x, size_t n, double* out);
int    rto_sum_dim(const float* x, const size_t* shape, size_t ndim, size_t dim, float* out);
int    rto_mean_dim(const float* x, const size_t* shape, size_t ndim, size_t dim, float* out);
/* max along a dim: no reference counterpart (the reference has no max_dim);
 * defined as the reference's global-max fold applied to each lane. */
int    rto_max_dim(const float* x, const size_t* shape, size_t ndim, size_t dim, float* out);

/* ---- optimizer rules: core/src/ops/optimizer.rs ---- */
int rto_adam_update(const float* p, const float* g, const float* m, const float* v, size_t n,
                    double lr, double beta1, double beta2, double eps, uint64_t t,
                    float* p_out, float* m_out, float* v_out);
int rto_adamw_update(const float* p, const float* g, const float* m, const float* v, size_t n,
                     double lr, double beta1, double beta2, double eps, double weight_decay,
                     uint64_t t, float* p_out, float* m_out, float* v_out);
int rto_sgd_update(const float* p, const float* g, size_t n, double lr, float* p_out);
int rto_sgd_momentum_update(const float* p, const float* g, const float* vel, size_t n,
                            double lr, double momentum, float* p_out, float* vel_out);

/* ---- nn optimizers: core/src/nn/optim.rs (f32 hyperparameters) ---- */
/* Adam::step (:262-313) for one parameter; t is the step count after the
 * increment at :264. */
void rto_nn_adam_step(const float* p, const float* g, const float* m, const float* v, size_t n,
                      float lr, float beta1, float beta2, float eps, uint64_t t, float* p_out,
                      float* m_out, float* v_out);
/* SGD::step (:148-208) for one parameter; vel/vel_out are used only when
 * momentum > 0. */
void rto_nn_sgd_step(const float* p, const float* g, const float* vel, size_t n, float lr,
                     float momentum, float weight_decay, float* p_out, float* vel_out);

/* ---- broadcasting: core/src/ops/broadcast.rs:55-198 ----
 * op: 0 add, 1 sub, 2 mul, 3 div.  Returns RTO_BROADCAST_ERROR for shapes
 * that do not broadcast; out has the broadcast shape. */
int rto_broadcast_binary(int op, const float* a, const size_t* ashape, size_t andim,
                         const float* b, const size_t* bshape, size_t bndim, float* out);

/* ---- autograd backward: core/src/autograd/ops.rs GradFn::backward ----
 * Each restates the ops::* chain the reference's backward builds, one f32
 * rounding per op, in its order.  NULL ga/gb skip that gradient. */
void rto_relu_backward(const float* g, const float* x, float* out, size_t n);    /* :375-390 */
void rto_sigmoid_backward(const float* g, const float* y, float* out, size_t n); /* :419-431 */
void rto_tanh_backward(const float* g, const float* y, float* out, size_t n);    /* :460-472 */
void rto_gelu_backward(const float* g, const float* x, float* out, size_t n);    /* :3102-3125 */
void rto_autograd_gelu(const float* x, float* out, size_t n);                    /* :3131-3141 */
void rto_sub_backward(const float* g, float* ga, float* gb, size_t n);           /* :175-192 */
void rto_mul_backward(const float* g, const float* a, const float* b, float* ga, float* gb,
                      size_t n);                                                 /* :219-236 */
void rto_div_backward(const float* g, const float* a, const float* b, float* ga, float* gb,
                      size_t n);                                                 /* :267-290 */
/* SumBackward / MeanBackward (:501-552): Tensor::full(shape, v) with
 * v = (f32)(f64)g or (f32)((f64)g / n). */
void rto_fill_backward(float g, float* out, size_t n, int mean);
/* reduce_to_shape (:627-681): grad of shape gshape folded onto oshape. */
int rto_reduce_to_shape(const float* grad, const size_t* gshape, size_t gnd, float* out,
                        const size_t* oshape, size_t ond);

/* The two f32 sums the losses use, on their own: ndarray's sum() of a
 * contiguous array (unrolled_fold, eight chains) and Iterator::sum from init. */
float rto_unrolled_sum_f32(const float* x, size_t n);
float rto_chain_sum_f32(const float* x, size_t n, float init);

/* ---- loss functions: core/src/ops/loss.rs (f32 inputs) ----
 * Each returns the reference's f64 result: the f32 sum of the per-element
 * terms, as f64, divided by n.  mse/l1/smooth_l1 sum with ndarray's sum()
 * (unrolled_fold: eight chains); bce/ce with Iterator::sum::<f32>() (one
 * chain from -0.0).  Argument checks are the caller's. */
double rto_mse_loss(const float* p, const float* t, size_t n);                    /* :41-85 (f32 path :71-75) */
double rto_l1_loss(const float* p, const float* t, size_t n);                     /* :102-144 (:132-135) */
double rto_smooth_l1_loss(const float* p, const float* t, size_t n, double beta); /* :165-229 (:203-214) */
double rto_bce_loss(const float* p, const float* t, size_t n, double epsilon);    /* :249-315 (:283-294) */
double rto_ce_loss(const float* p, const float* t, size_t n, double epsilon);     /* :332-391 (:362-372) */

/* ---- seeded synthetic inputs (the generator the tests and the CPU baseline
 * use; the CUDA library carries an identical device generator).  Element i of
 * a stream depends only on (seed, i), so any slice can be regenerated alone.
 *   uniform: u = (splitmix64(seed, i) >> 40) * 2^-24 in [0,1); lo + (hi-lo)*u
 *   normal : Box-Muller in f64 on two 26-bit uniforms from one 64-bit draw  */
void rto_fill_uniform(float* out, size_t n, uint64_t seed, uint64_t offset, float lo, float hi);
void rto_fill_normal(float* out, size_t n, uint64_t seed, uint64_t offset, float mean, float std);

/* Threads used by the reference's rayon-parallel ops (add when n >= 10000);
 * defaults to the number of online CPUs, like rayon's global pool
 * (core/src/ffi/mod.rs:25-32).  0 restores the default. */
void rto_set_threads(int n);
int  rto_get_threads(void);

#ifdef __cplusplus
}
#endif
#endif
