// rt_internal.h — launchers shared between the kernel files and the C-ABI
// layer (abi.cu).  Nothing here is exported from the shared library.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace rt {

// Threads per block for the streaming kernels.
constexpr int kThreads = 256;

// Number of SMs of `device` (cached after the first query).
int sm_count(int device);

// ------------------------------------------------------------------ math mode
// Whether the transcendental activations and softmax reproduce glibc's bits
// (exact) or stay within 1e-6 relative error / 4 ulp of them (tolerance, the
// default).  Process-wide; the RTC_MATH_MODE environment variable ("exact" or
// "tolerance") sets the initial value.
bool math_exact();
void set_math_exact(bool exact);

// ---------------------------------------------------------------- elementwise
enum UnaryOp {
  kRelu, kLeakyRelu, kSigmoid, kTanh, kGelu, kSwish, kElu, kSelu, kMish, kSoftplus, kSoftsign,
  kAddScalar, kMulScalar,
};
enum BinaryOp { kAdd, kSub, kMul, kDiv, kAddMulScalar };

// `param` is alpha (leaky_relu, elu) or the scalar (add/mul_scalar).
cudaError_t launch_unary(UnaryOp op, float param, const float* x, float* out, size_t n,
                         cudaStream_t s);
cudaError_t launch_binary(BinaryOp op, float param, const float* a, const float* b, float* out,
                          size_t n, cudaStream_t s);
cudaError_t launch_fma(const float* a, const float* b, const float* c, float* out, size_t n,
                       cudaStream_t s);

// Coefficients of one Adam/AdamW step, already rounded to f32 on the host
// exactly as rusttorch-core rounds them (optimizer.rs:278-309, :413-418).
struct AdamCoeffs {
  float b1, one_minus_b1, b2, one_minus_b2, bc1, bc2, eps, lr;
  float lr_wd;      // (f32)(lr*wd) in f64; used only when decay != 0
  int decay;        // weight_decay > 0
};
cudaError_t launch_adam(const float* p, const float* g, const float* m, const float* v,
                        float* p_out, float* m_out, float* v_out, size_t n, const AdamCoeffs& c,
                        cudaStream_t s);
cudaError_t launch_sgd(const float* p, const float* g, float* p_out, size_t n, float lr,
                       cudaStream_t s);
cudaError_t launch_sgd_momentum(const float* p, const float* g, const float* vel, float* p_out,
                                float* vel_out, size_t n, float lr, float momentum,
                                cudaStream_t s);

// nn::Adam::step coefficients (core/src/nn/optim.rs:262-313): f32 throughout,
// bias corrections 1 - powf(beta, t) in f32.
struct NnAdamCoeffs {
  float b1, one_minus_b1, b2, one_minus_b2, bc1, bc2, lr, eps;
};
cudaError_t launch_nn_adam(const float* p, const float* g, const float* m, const float* v,
                           float* p_out, float* m_out, float* v_out, size_t n,
                           const NnAdamCoeffs& c, cudaStream_t s);
// nn::SGD::step (core/src/nn/optim.rs:148-208); vel/vel_out only when
// momentum > 0.
cudaError_t launch_nn_sgd(const float* p, const float* g, const float* vel, float* p_out,
                          float* vel_out, size_t n, float lr, float momentum, float wd,
                          cudaStream_t s);

// Broadcast binary op (core/src/ops/broadcast.rs:177-198) on C-contiguous
// inputs; dims already collapsed: out has shape[0..nd), a and b element
// strides per dim (0 where broadcast).
constexpr int kMaxBcastDims = 8;
struct BcastPlan {
  int nd;
  long long shape[kMaxBcastDims];
  long long astride[kMaxBcastDims];
  long long bstride[kMaxBcastDims];
};
cudaError_t launch_broadcast(BinaryOp op, const float* a, const float* b, float* out,
                             size_t n, const BcastPlan& plan, cudaStream_t s);

// ----------------------------------------------------------------- reductions
// Per-block partial of the one-pass global statistics.  `mx`/`mn` ignore NaN
// (fmaxf/fminf); the caller repairs the rare cases in which the reference's
// fold gives a different bit pattern (NaN present, or a zero extreme).
struct StatsPart {
  double sum;
  float mx;
  float mn;
};
// Blocks used by launch_stats on `device` for n elements (<= stats_max_parts).
int stats_num_parts(int device, size_t n);
int stats_max_parts(int device);
// Writes the combined statistics of x[0..n) to *out (device memory, may be
// null) and the sum alone to *sum_out (device memory, may be null).
// `parts` is scratch of stats_num_parts(device, n) entries.
cudaError_t launch_stats(const float* x, size_t n, StatsPart* parts, int nparts, StatsPart* out,
                         cudaStream_t s, double* sum_out = nullptr);

// launch_stats with another kernel shape (threads 256/512/1024, U loads in
// flight per thread, blocks_per_sm <= 0: as many as stay resident) and at
// most max_parts partials; the sum alone goes to *sum_out.  For the probes.
cudaError_t launch_stats_variant(int threads, int u, int blocks_per_sm, const float* x, size_t n,
                                 StatsPart* parts, int max_parts, cudaStream_t s,
                                 double* sum_out);

// The grid-stride, software-pipelined stats kernel (threads 256/512, u 2/4).
cudaError_t launch_stats_gs_variant(int threads, int u, int blocks_per_sm, const float* x,
                                    size_t n, StatsPart* parts, int max_parts, cudaStream_t s,
                                    double* sum_out);

// The last-axis sum of [lanes, len] (len % 4 == 0, 16-byte-aligned x) by
// the four-lanes-per-warp kernel with `warps` (1, 2, 4, 8) warps per CTA.
// For the probes.
cudaError_t launch_lane_sum_variant(int warps, const float* x, size_t lanes, size_t len,
                                    float* out, cudaStream_t s);

// Positions used by the exact repair path, 1-based (0 = none).
struct IndexScan {
  unsigned long long last_nan;    // last i+1 with x[i] NaN
  unsigned long long first_zero;  // first i+1 with x[i] == 0 (~0ull = none)
  unsigned long long last_zero;   // last i+1 with x[i] == 0
};
cudaError_t launch_index_scan(const float* x, size_t n, IndexScan* out, cudaStream_t s);

enum DimReduce { kDimSum, kDimMean, kDimMax };
// Reduce the middle axis of a C-contiguous [outer, len, inner] tensor.
// `last_axis`: the reduced axis is the tensor's last axis, which ndarray's
// sum_axis reduces lane by lane with the eight-chain unrolled_fold (its
// minimum-stride axis; default strides make that the last axis even when the
// axes after `dim` all have length 1).  Any other axis is summed as one
// row-order chain per output from 0.0 — with inner == 1 too.
cudaError_t launch_reduce_dim(DimReduce op, const float* x, size_t outer, size_t len,
                              size_t inner, bool last_axis, float* out, cudaStream_t s);
// The TMA-staged variant for inner > 1 (strip_tma.cu).  Sets *used = false
// (and launches nothing) when the layout does not suit TMA.
cudaError_t launch_strip_tma(DimReduce op, const float* x, size_t outer, size_t len,
                             size_t inner, float* out, cudaStream_t s, bool* used);
// The same with the strip shape given: W columns per CTA (a multiple of 4),
// R rows per tile, `stages` tiles in the ring; fixed_width: W = 16 and 32
// use kernels compiled for that width (bench.py's sizing probe compares).
cudaError_t launch_strip_tma_shape(DimReduce op, const float* x, size_t outer, size_t len,
                                   size_t inner, float* out, cudaStream_t s, bool* used,
                                   size_t W, size_t R, int stages, bool fixed_width);

// ------------------------------------------------------- autograd backward
enum GradUnaryOp { kGradRelu, kGradSigmoid, kGradTanh, kGradGelu };
enum GradBinaryOp { kGradAdd, kGradSub, kGradMul, kGradDiv };
// out = dL/dx from grad_output g and the saved input (relu, gelu) or output
// (sigmoid, tanh).
cudaError_t launch_grad_unary(GradUnaryOp op, const float* g, const float* saved, float* out,
                              size_t n, cudaStream_t s);
// grad_a / grad_b may be null (that operand needs no gradient); a and b are
// read only by mul and div.
cudaError_t launch_grad_binary(GradBinaryOp op, const float* g, const float* a, const float* b,
                               float* grad_a, float* grad_b, size_t n, cudaStream_t s);
// autograd's own gelu forward (autograd/ops.rs:3131), which rounds
// differently from ops::gelu.
cudaError_t launch_gelu_autograd(const float* x, float* out, size_t n, cudaStream_t s);
// out[0..n) = (f32)(f64)g[0], or (f32)((f64)g[0] / divisor) when `divide`.
cudaError_t launch_fill_from(const float* g, float* out, size_t n, double divisor, bool divide,
                             cudaStream_t s);
// Each contiguous lane of length len summed as one sequential f32 chain from
// 0.0, in element order; with `mean`, the chain's value / (f32)len.
cudaError_t launch_lane_chain_sum(const float* x, size_t lanes, size_t len, float* out,
                                  cudaStream_t s, bool mean = false);
// sqrt(2/pi) as the reference computes it in f32.
float gelu_k();

// ------------------------------------------------------------------- losses
enum LossOp { kLossMse, kLossL1, kLossSmoothL1, kLossBce, kLossCe };
// *sum_out (device) = the reference's ordered f32 sum of the loss terms of
// p and t; `scratch` is loss_scratch_bytes(op, n) bytes of 256-byte-aligned
// device memory.  a, b: smooth_l1 (beta, 0.5*beta), bce (eps, 1 - eps), ce
// (eps, unused), in f32.
size_t loss_scratch_bytes(LossOp op, size_t n);
cudaError_t launch_loss(LossOp op, const float* p, const float* t, size_t n, float a, float b,
                        void* scratch, float* sum_out, cudaStream_t s);
// *sum_out (device) = x's ordered f32 sum: ndarray's unrolled_fold for
// chains == 8, init + x[0] + x[1] + ... for chains == 1.  Scratch as for a
// loss of the same chain count.
cudaError_t launch_ordered_sum_of(const float* x, size_t n, int chains, float init, void* scratch,
                                  float* sum_out, cudaStream_t s);
// Bytes of scratch launch_ordered_sum_of needs for n terms in `chains` chains.
size_t ordered_sum_scratch_bytes(size_t n, int chains);

// -------------------------------------------------------------------- softmax
// last_axis as for launch_reduce_dim: it picks the order of the sum of exps.
cudaError_t launch_softmax(const float* x, size_t outer, size_t len, size_t inner,
                           bool last_axis, float* out, cudaStream_t s);

// ------------------------------------------------------------------ generator
cudaError_t launch_fill(float* out, size_t n, uint64_t seed, uint64_t offset, float a, float b,
                        int normal, cudaStream_t s);

}  // namespace rt
