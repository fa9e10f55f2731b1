// abi_loss.cu — C-ABI entry points for rusttorch-core's loss functions
// (src/ops/loss.rs).  The reference exposes them only as Rust functions
// returning Result<f64>; here each returns that f64 through out_value.
// Argument checks follow each function's own order and messages.  f32
// tensors on a device are computed (f64 tensors: RTC_UNSUPPORTED after the
// reference's checks; host tensors: RTC_INVALID_ARGUMENT).
#include "rt_abi_util.h"

using namespace rt;

namespace {

// loss.rs:43-67 (mse, l1; smooth_l1 adds its beta check after dtype):
// shape (expected targets, got predictions), then dtype, then emptiness.
rtc_result shape_dtype(const rtc_tensor* p, const rtc_tensor* t, const char* ctx,
                       bool check_dtype) {
  TRY(check_desc(p, "predictions"));
  TRY(check_desc(t, "targets"));
  if (!same_shape(p, t)) return shape_mismatch(ctx, t, p);
  if (check_dtype && p->dtype != t->dtype)
    return dtype_mismatch(ctx, dtype_display(t->dtype), dtype_display(p->dtype));
  return ok();
}

// The f32/f64 match arm (e.g. loss.rs:70-84): anything else is a dtype error.
rtc_result float_pair(const rtc_tensor* p, const rtc_tensor* t, const char* ctx) {
  const bool f32 = p->dtype == RTC_F32 && t->dtype == RTC_F32;
  const bool f64 = p->dtype == RTC_F64 && t->dtype == RTC_F64;
  if (!f32 && !f64)
    return dtype_mismatch(std::string(ctx) + " (only floating-point supported)",
                          "float32 or float64", dtype_display(p->dtype));
  TRY(require_f32(p, ctx));
  if (p->device == RTC_HOST_MEMORY || t->device == RTC_HOST_MEMORY)
    return invalid_argument("device", std::string(ctx) + " needs device tensors");
  TRY(same_device(p, t, t));
  return ok();
}

rtc_result run_loss(LossOp op, const rtc_tensor* p, const rtc_tensor* t, float a, float b,
                    const char* ctx, double* out_value) {
  const size_t n = p->numel;
  DeviceScope scope(p->device);
  if (!scope.ok()) return backend_error("cudaSetDevice", scope.error());
  cudaStream_t s = thread_stream();
  keep_pool_memory(p->device);
  const size_t scratch_bytes = loss_scratch_bytes(op, n);
  char* scratch = nullptr;
  cudaError_t e = cudaMallocAsync(reinterpret_cast<void**>(&scratch), scratch_bytes + 256, s);
  if (e != cudaSuccess) return backend_error(ctx, e);
  float* sum_dev = reinterpret_cast<float*>(scratch + scratch_bytes);
  float sum = 0.0f;
  e = launch_loss(op, cf(p), cf(t), n, a, b, scratch, sum_dev, s);
  if (e == cudaSuccess) e = cudaMemcpyAsync(&sum, sum_dev, sizeof sum, cudaMemcpyDeviceToHost, s);
  const cudaError_t ef = cudaFreeAsync(scratch, s);
  if (e == cudaSuccess) e = ef;
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return backend_error(ctx, e);
  *out_value = (double)sum / (double)n;
  return ok();
}

}  // namespace

extern "C" rtc_result rtc_mse_loss(const rtc_tensor* predictions, const rtc_tensor* targets,
                                   double* out_value) {
  RTC_OP_RANGE();
  const char* ctx = "mse_loss";
  if (!out_value) return invalid_argument("out_value", "must not be null");
  TRY(shape_dtype(predictions, targets, ctx, true));
  if (predictions->numel == 0) return empty_tensor(ctx);
  TRY(float_pair(predictions, targets, ctx));
  return run_loss(kLossMse, predictions, targets, 0.0f, 0.0f, ctx, out_value);
}

extern "C" rtc_result rtc_l1_loss(const rtc_tensor* predictions, const rtc_tensor* targets,
                                  double* out_value) {
  RTC_OP_RANGE();
  const char* ctx = "l1_loss";
  if (!out_value) return invalid_argument("out_value", "must not be null");
  TRY(shape_dtype(predictions, targets, ctx, true));
  if (predictions->numel == 0) return empty_tensor(ctx);
  TRY(float_pair(predictions, targets, ctx));
  return run_loss(kLossL1, predictions, targets, 0.0f, 0.0f, ctx, out_value);
}

// loss.rs:182-188: `beta <= 0.0` (a NaN beta passes)
extern "C" rtc_result rtc_smooth_l1_loss(const rtc_tensor* predictions, const rtc_tensor* targets,
                                         double beta, double* out_value) {
  RTC_OP_RANGE();
  const char* ctx = "smooth_l1_loss";
  if (!out_value) return invalid_argument("out_value", "must not be null");
  TRY(shape_dtype(predictions, targets, ctx, true));
  if (beta <= 0.0) return invalid_argument("beta", "must be positive, got " + rust_f64(beta));
  if (predictions->numel == 0) return empty_tensor(ctx);
  TRY(float_pair(predictions, targets, ctx));
  const float bf = (float)beta;
  volatile float half = 0.5f;
  return run_loss(kLossSmoothL1, predictions, targets, bf, half * bf, ctx, out_value);
}

// loss.rs:254-273 / :333-352: shape, then epsilon in (0, 1), then emptiness;
// no separate dtype check (the match arm rejects mixed dtypes).
static rtc_result xent(LossOp op, const rtc_tensor* p, const rtc_tensor* t, double epsilon,
                       const char* ctx, double* out_value) {
  if (!out_value) return invalid_argument("out_value", "must not be null");
  TRY(shape_dtype(p, t, ctx, false));
  if (epsilon <= 0.0 || epsilon >= 1.0)
    return invalid_argument("epsilon", "must be in (0, 1), got " + rust_f64(epsilon));
  if (p->numel == 0) return empty_tensor(ctx);
  TRY(float_pair(p, t, ctx));
  const float ef = (float)epsilon;
  volatile float one = 1.0f;
  return run_loss(op, p, t, ef, one - ef, ctx, out_value);
}

extern "C" rtc_result rtc_binary_cross_entropy_loss(const rtc_tensor* predictions,
                                                    const rtc_tensor* targets, double epsilon,
                                                    double* out_value) {
  RTC_OP_RANGE();
  return xent(kLossBce, predictions, targets, epsilon, "binary_cross_entropy_loss", out_value);
}

extern "C" rtc_result rtc_cross_entropy_loss(const rtc_tensor* predictions,
                                             const rtc_tensor* targets, double epsilon,
                                             double* out_value) {
  RTC_OP_RANGE();
  return xent(kLossCe, predictions, targets, epsilon, "cross_entropy_loss", out_value);
}

// Test hook (no reference counterpart): *out_value = the ordered f32 sum of
// x's elements, ndarray's unrolled_fold for chains == 8, init + x[0] + x[1]
// + ... for chains == 1 — the sums that the losses above reproduce.
extern "C" rtc_result rtc_selftest_ordered_sum(const rtc_tensor* x, int chains, float init,
                                               float* out_value) {
  RTC_OP_RANGE();
  const char* ctx = "selftest_ordered_sum";
  if (!out_value) return invalid_argument("out_value", "must not be null");
  TRY(check_desc(x, "x"));
  if (chains != 1 && chains != 8) return invalid_argument("chains", "must be 1 or 8");
  TRY(require_f32(x, ctx));
  if (x->device == RTC_HOST_MEMORY) return invalid_argument("device", "needs a device tensor");
  const size_t n = x->numel;
  if (n == 0) {
    *out_value = chains == 8 ? 0.0f : init;
    return ok();
  }
  DeviceScope scope(x->device);
  if (!scope.ok()) return backend_error("cudaSetDevice", scope.error());
  cudaStream_t s = thread_stream();
  keep_pool_memory(x->device);
  const size_t scratch_bytes = loss_scratch_bytes(chains == 8 ? kLossMse : kLossBce, n);
  char* scratch = nullptr;
  cudaError_t e = cudaMallocAsync(reinterpret_cast<void**>(&scratch), scratch_bytes + 256, s);
  if (e != cudaSuccess) return backend_error(ctx, e);
  float* sum_dev = reinterpret_cast<float*>(scratch + scratch_bytes);
  float sum = 0.0f;
  e = launch_ordered_sum_of(cf(x), n, chains, init, scratch, sum_dev, s);
  if (e == cudaSuccess) e = cudaMemcpyAsync(&sum, sum_dev, sizeof sum, cudaMemcpyDeviceToHost, s);
  const cudaError_t ef = cudaFreeAsync(scratch, s);
  if (e == cudaSuccess) e = ef;
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return backend_error(ctx, e);
  *out_value = sum;
  return ok();
}
