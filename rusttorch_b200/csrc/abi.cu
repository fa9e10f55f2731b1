// abi.cu — the exported C ABI (include/rusttorch_cuda.h).
//
// Each entry point validates its arguments on the host in the order the
// reference does (so that the first error reported is the reference's), with
// the reference's error text (rusttorch-core/src/error.rs:69-160), then checks
// what the device path itself needs (consistent descriptors, contiguity,
// float32) and launches on the calling thread's stream.  Nothing here touches
// the CUDA runtime before validation has passed, so every error path works on
// a machine without a GPU.
#include "../../include/rusttorch_cuda.h"
#include "rt_abi_util.h"
#include "rt_tma.cuh"
#include "rt_internal.h"
#include "rt_staging.h"

#include <algorithm>
#include <thread>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

using namespace rt;

// ------------------------------------------------------------------ lifecycle

extern "C" const char* rtc_version(void) { return RTC_VERSION_STRING; }

extern "C" rtc_result rtc_init(void) {
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess) return backend_error("cudaGetDeviceCount", e);
  for (int d = 0; d < n; d++) {
    DeviceScope scope(d);
    e = cudaFree(nullptr);
    if (e != cudaSuccess) return backend_error("cudaFree(0)", e);
    keep_pool_memory(d);
  }
  return ok();
}

extern "C" void rtc_cleanup(void) { release_library_state(); }

extern "C" void rtc_free_error_message(char* msg) { std::free(msg); }

extern "C" rtc_result rtc_set_stream(void* stream) {
  set_thread_stream(static_cast<cudaStream_t>(stream));
  return ok();
}

extern "C" void* rtc_get_stream(void) { return static_cast<void*>(thread_stream()); }

extern "C" rtc_result rtc_synchronize(void) {
  cudaError_t e = cudaStreamSynchronize(thread_stream());
  if (e != cudaSuccess) return backend_error("cudaStreamSynchronize", e);
  int device = 0;
  cudaGetDevice(&device);
  if (take_wait_timeouts(device))
    return fail(RTC_BACKEND_ERROR,
                "a kernel gave up waiting (for a shared-memory tile or another rank; "
                "2 s limit); results since the last synchronize are incomplete");
  return ok();
}

extern "C" rtc_result rtc_selftest_bounded_wait(void) {
  int device = 0;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess) return backend_error("cudaGetDevice", e);
  return launched(launch_bounded_wait_probe(device, thread_stream()), "selftest_bounded_wait");
}

extern "C" rtc_result rtc_set_math_mode(int mode) {
  if (mode != RTC_MATH_TOLERANCE && mode != RTC_MATH_EXACT)
    return invalid_argument("mode", "must be RTC_MATH_TOLERANCE or RTC_MATH_EXACT");
  set_math_exact(mode == RTC_MATH_EXACT);
  return ok();
}

extern "C" int rtc_get_math_mode(void) { return math_exact() ? RTC_MATH_EXACT : RTC_MATH_TOLERANCE; }

extern "C" int rtc_device_count(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) return 0;
  return n;
}

extern "C" rtc_result rtc_set_device(int device) {
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return backend_error("cudaSetDevice", e);
  return ok();
}

extern "C" int rtc_get_device(void) {
  int d = 0;
  if (cudaGetDevice(&d) != cudaSuccess) return -1;
  return d;
}

static bool on_host(const rtc_tensor* t) { return t->device == RTC_HOST_MEMORY; }

// ---------------------------------------------------------------- memory

extern "C" rtc_result rtc_malloc(int device, size_t bytes, void** out) {
  RTC_OP_RANGE();
  if (!out) return invalid_argument("out", "must not be null");
  *out = nullptr;
  if (bytes == 0) return ok();
  DeviceScope scope(device);
  if (!scope.ok()) return backend_error("cudaSetDevice", scope.error());
  cudaError_t e = cudaMalloc(out, bytes);
  if (e != cudaSuccess) return backend_error("cudaMalloc", e);
  return ok();
}

extern "C" rtc_result rtc_free(int device, void* ptr) {
  RTC_OP_RANGE();
  if (!ptr) return ok();
  DeviceScope scope(device);
  if (!scope.ok()) return backend_error("cudaSetDevice", scope.error());
  cudaError_t e = cudaFree(ptr);
  if (e != cudaSuccess) return backend_error("cudaFree", e);
  return ok();
}

extern "C" rtc_result rtc_memcpy_h2d(int device, void* dst, const void* src, size_t bytes) {
  RTC_OP_RANGE();
  if (bytes == 0) return ok();
  if (!dst || !src) return invalid_argument("pointer", "must not be null");
  DeviceScope scope(device);
  if (!scope.ok()) return backend_error("cudaSetDevice", scope.error());
  cudaStream_t s = thread_stream();
  cudaError_t e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return backend_error("cudaMemcpyAsync(H2D)", e);
  return ok();
}

extern "C" rtc_result rtc_memcpy_d2h(int device, void* dst, const void* src, size_t bytes) {
  RTC_OP_RANGE();
  if (bytes == 0) return ok();
  if (!dst || !src) return invalid_argument("pointer", "must not be null");
  DeviceScope scope(device);
  if (!scope.ok()) return backend_error("cudaSetDevice", scope.error());
  cudaStream_t s = thread_stream();
  cudaError_t e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return backend_error("cudaMemcpyAsync(D2H)", e);
  return ok();
}

extern "C" rtc_result rtc_host_alloc(size_t bytes, void** out) {
  RTC_OP_RANGE();
  if (!out) return invalid_argument("out", "must not be null");
  *out = nullptr;
  if (bytes == 0) return ok();
  cudaError_t e = cudaHostAlloc(out, bytes, cudaHostAllocPortable);
  if (e != cudaSuccess) return backend_error("cudaHostAlloc", e);
  return ok();
}

extern "C" rtc_result rtc_host_free(void* ptr) {
  RTC_OP_RANGE();
  if (!ptr) return ok();
  cudaError_t e = cudaFreeHost(ptr);
  if (e != cudaSuccess) return backend_error("cudaFreeHost", e);
  return ok();
}

// ----------------------------------------------------------------- generator

static rtc_result fill(const rtc_tensor* out, uint64_t seed, uint64_t offset, float a, float b,
                       int normal) {
  TRY(check_desc(out, "out"));
  TRY(require_f32(out, normal ? "fill_normal" : "fill_uniform"));
  if (out->numel == 0) return ok();
  DeviceScope scope(out->device);
  if (!scope.ok()) return backend_error("cudaSetDevice", scope.error());
  return launched(launch_fill(static_cast<float*>(out->data), out->numel, seed, offset, a, b,
                              normal, thread_stream()),
                  "fill");
}

extern "C" rtc_result rtc_fill_uniform(const rtc_tensor* out, uint64_t seed, uint64_t offset,
                                       float lo, float hi) {
  RTC_OP_RANGE();
  return fill(out, seed, offset, lo, hi, 0);
}

extern "C" rtc_result rtc_fill_normal(const rtc_tensor* out, uint64_t seed, uint64_t offset,
                                      float mean, float std) {
  RTC_OP_RANGE();
  return fill(out, seed, offset, mean, std, 1);
}

// --------------------------------------------------------------- elementwise

// Binary ops: the reference checks dtype, then shape (elementwise.rs:15-28);
// div also requires a float dtype (:178-183).
static rtc_result binary(BinaryOp op, float param, const rtc_tensor* a, const rtc_tensor* b,
                         const rtc_tensor* out, const char* context, bool float_only,
                         const char* float_reason) {
  TRY(check_desc(a, "a"));
  TRY(check_desc(b, "b"));
  TRY(check_desc(out, "out"));
  if (a->dtype != b->dtype)
    return dtype_mismatch(context, dtype_debug(a->dtype), dtype_debug(b->dtype));
  if (!same_shape(a, b)) return shape_mismatch(context, a, b);
  if (float_only && !is_float(a->dtype)) return invalid_argument("dtype", float_reason);
  TRY(check_output(a, out, context));
  TRY(require_f32(a, context));
  TRY(same_device(a, b, out));
  if (a->numel == 0) return ok();
  if (on_host(a)) {
    const std::vector<size_t> iu{4, 4}, ou{4};
    const std::vector<int> al{-1};
    return launched(staged_map({a->data, b->data}, iu, {out->data}, ou, al, a->numel,
                               staged_chunk_units(iu, ou, al),
                               [=](const void* const* din, void* const* dout, size_t, size_t cu,
                                   cudaStream_t s) {
                                 return launch_binary(op, param, (const float*)din[0],
                                                      (const float*)din[1], (float*)dout[0], cu, s);
                               }),
                    context);
  }
  DeviceScope scope(a->device);
  if (!scope.ok()) return backend_error("cudaSetDevice", scope.error());
  return launched(launch_binary(op, param, cf(a), cf(b), f(out), a->numel, thread_stream()),
                  context);
}

extern "C" rtc_result rtc_add(const rtc_tensor* a, const rtc_tensor* b, const rtc_tensor* out) {
  RTC_OP_RANGE();
  return binary(kAdd, 0.f, a, b, out, "element-wise addition", false, nullptr);
}
extern "C" rtc_result rtc_mul(const rtc_tensor* a, const rtc_tensor* b, const rtc_tensor* out) {
  RTC_OP_RANGE();
  return binary(kMul, 0.f, a, b, out, "element-wise multiplication", false, nullptr);
}
extern "C" rtc_result rtc_sub(const rtc_tensor* a, const rtc_tensor* b, const rtc_tensor* out) {
  RTC_OP_RANGE();
  return binary(kSub, 0.f, a, b, out, "element-wise subtraction", false, nullptr);
}
extern "C" rtc_result rtc_div(const rtc_tensor* a, const rtc_tensor* b, const rtc_tensor* out) {
  RTC_OP_RANGE();
  return binary(kDiv, 0.f, a, b, out, "element-wise division", true,
                "Division requires floating-point tensors");
}
extern "C" rtc_result rtc_add_simd(const rtc_tensor* a, const rtc_tensor* b,
                                   const rtc_tensor* out) {
  RTC_OP_RANGE();
  return binary(kAdd, 0.f, a, b, out, "add_simd", false, nullptr);
}
extern "C" rtc_result rtc_mul_simd(const rtc_tensor* a, const rtc_tensor* b,
                                   const rtc_tensor* out) {
  RTC_OP_RANGE();
  return binary(kMul, 0.f, a, b, out, "mul_simd", false, nullptr);
}
// ops::add then ops::mul_scalar: add's checks apply (mul_scalar has none).
extern "C" rtc_result rtc_add_mul_scalar(const rtc_tensor* a, const rtc_tensor* b, float scalar,
                                         const rtc_tensor* out) {
  RTC_OP_RANGE();
  return binary(kAddMulScalar, scalar, a, b, out, "element-wise addition", false, nullptr);
}

// simd.rs:276-297 checks shapes first, then dtypes, and needs floats (:361-366).
extern "C" rtc_result rtc_fused_multiply_add(const rtc_tensor* a, const rtc_tensor* b,
                                             const rtc_tensor* c, const rtc_tensor* out) {
  RTC_OP_RANGE();
  const char* context = "fused_multiply_add";
  TRY(check_desc(a, "a"));
  TRY(check_desc(b, "b"));
  TRY(check_desc(c, "c"));
  TRY(check_desc(out, "out"));
  if (!same_shape(a, b)) return shape_mismatch(context, a, b);
  if (!same_shape(a, c)) return shape_mismatch(context, a, c);
  if (a->dtype != b->dtype)
    return dtype_mismatch(context, dtype_debug(a->dtype), dtype_debug(b->dtype));
  if (a->dtype != c->dtype)
    return dtype_mismatch(context, dtype_debug(a->dtype), dtype_debug(c->dtype));
  if (!is_float(a->dtype))
    return invalid_argument("dtype", "fused_multiply_add only supports floating-point tensors");
  TRY(check_output(a, out, context));
  TRY(require_f32(a, context));
  TRY(same_device(a, b, out));
  TRY(same_device(a, c, out));
  if (a->numel == 0) return ok();
  if (on_host(a)) {
    const std::vector<size_t> iu{4, 4, 4}, ou{4};
    const std::vector<int> al{-1};
    return launched(staged_map({a->data, b->data, c->data}, iu, {out->data}, ou, al, a->numel,
                               staged_chunk_units(iu, ou, al),
                               [](const void* const* din, void* const* dout, size_t, size_t cu,
                                  cudaStream_t s) {
                                 return launch_fma((const float*)din[0], (const float*)din[1],
                                                   (const float*)din[2], (float*)dout[0], cu, s);
                               }),
                    context);
  }
  DeviceScope scope(a->device);
  if (!scope.ok()) return backend_error("cudaSetDevice", scope.error());
  return launched(launch_fma(cf(a), cf(b), cf(c), f(out), a->numel, thread_stream()), context);
}

// Unary ops.  `float_reason` set: the op rejects integer tensors first
// (activation.rs:22-27 and the like); otherwise every dtype is accepted by the
// reference.
static rtc_result unary(UnaryOp op, float param, const rtc_tensor* x, const rtc_tensor* out,
                        const char* context, const char* float_reason) {
  TRY(check_desc(x, "input"));
  TRY(check_desc(out, "out"));
  if (float_reason && !is_float(x->dtype)) return invalid_argument("dtype", float_reason);
  // activation.rs:202: `if alpha <= 0.0` (so a NaN alpha passes)
  if (op == kElu && param <= 0.0f) return invalid_argument("alpha", "Alpha must be positive");
  TRY(check_output(x, out, context));
  TRY(require_f32(x, context));
  TRY(same_device(x, out, out));
  if (x->numel == 0) return ok();
  if (on_host(x)) {
    const std::vector<size_t> iu{4}, ou{4};
    const std::vector<int> al{-1};
    return launched(staged_map({x->data}, iu, {out->data}, ou, al, x->numel,
                               staged_chunk_units(iu, ou, al),
                               [=](const void* const* din, void* const* dout, size_t, size_t cu,
                                   cudaStream_t s) {
                                 return launch_unary(op, param, (const float*)din[0],
                                                     (float*)dout[0], cu, s);
                               }),
                    context);
  }
  DeviceScope scope(x->device);
  if (!scope.ok()) return backend_error("cudaSetDevice", scope.error());
  return launched(launch_unary(op, param, cf(x), f(out), x->numel, thread_stream()), context);
}

extern "C" rtc_result rtc_add_scalar(const rtc_tensor* x, float s, const rtc_tensor* out) {
  RTC_OP_RANGE();
  return unary(kAddScalar, s, x, out, "add_scalar", nullptr);
}
extern "C" rtc_result rtc_mul_scalar(const rtc_tensor* x, float s, const rtc_tensor* out) {
  RTC_OP_RANGE();
  return unary(kMulScalar, s, x, out, "mul_scalar", nullptr);
}
extern "C" rtc_result rtc_mul_scalar_simd(const rtc_tensor* x, float s, const rtc_tensor* out) {
  RTC_OP_RANGE();
  return unary(kMulScalar, s, x, out, "mul_scalar_simd", nullptr);
}
extern "C" rtc_result rtc_relu(const rtc_tensor* x, const rtc_tensor* out) {
  RTC_OP_RANGE();
  return unary(kRelu, 0.f, x, out, "relu", nullptr);
}
extern "C" rtc_result rtc_relu_simd(const rtc_tensor* x, const rtc_tensor* out) {
  RTC_OP_RANGE();
  return unary(kRelu, 0.f, x, out, "relu_simd", nullptr);
}
extern "C" rtc_result rtc_leaky_relu(const rtc_tensor* x, const rtc_tensor* out, float alpha) {
  RTC_OP_RANGE();
  return unary(kLeakyRelu, alpha, x, out, "leaky_relu", nullptr);
}
extern "C" rtc_result rtc_sigmoid(const rtc_tensor* x, const rtc_tensor* out) {
  RTC_OP_RANGE();
  return unary(kSigmoid, 0.f, x, out, "sigmoid", "Sigmoid requires floating-point tensors");
}
extern "C" rtc_result rtc_tanh(const rtc_tensor* x, const rtc_tensor* out) {
  RTC_OP_RANGE();
  return unary(kTanh, 0.f, x, out, "tanh", "Tanh requires floating-point tensors");
}
extern "C" rtc_result rtc_gelu(const rtc_tensor* x, const rtc_tensor* out) {
  RTC_OP_RANGE();
  return unary(kGelu, 0.f, x, out, "gelu", "GELU requires floating-point tensors");
}
extern "C" rtc_result rtc_swish(const rtc_tensor* x, const rtc_tensor* out) {
  RTC_OP_RANGE();
  return unary(kSwish, 0.f, x, out, "swish", "Swish requires floating-point tensors");
}
extern "C" rtc_result rtc_elu(const rtc_tensor* x, const rtc_tensor* out, float alpha) {
  RTC_OP_RANGE();
  return unary(kElu, alpha, x, out, "elu", "ELU requires floating-point tensors");
}
extern "C" rtc_result rtc_selu(const rtc_tensor* x, const rtc_tensor* out) {
  RTC_OP_RANGE();
  return unary(kSelu, 0.f, x, out, "selu", "SELU requires floating-point tensors");
}
extern "C" rtc_result rtc_mish(const rtc_tensor* x, const rtc_tensor* out) {
  RTC_OP_RANGE();
  return unary(kMish, 0.f, x, out, "mish", "Mish requires floating-point tensors");
}
extern "C" rtc_result rtc_softplus(const rtc_tensor* x, const rtc_tensor* out) {
  RTC_OP_RANGE();
  return unary(kSoftplus, 0.f, x, out, "softplus", "Softplus requires floating-point tensors");
}
extern "C" rtc_result rtc_softsign(const rtc_tensor* x, const rtc_tensor* out) {
  RTC_OP_RANGE();
  return unary(kSoftsign, 0.f, x, out, "softsign", "Softsign requires floating-point tensors");
}

extern "C" rtc_result rtc_relu_f32(const float* input, float* output, size_t size) {
  RTC_OP_RANGE();
  if (size == 0) return ok();
  if (!input || !output) return invalid_argument("pointer", "must not be null");
  return launched(launch_unary(kRelu, 0.f, input, output, size, thread_stream()), "relu_f32");
}
extern "C" rtc_result rtc_add_f32(const float* a, const float* b, float* output, size_t size) {
  RTC_OP_RANGE();
  if (size == 0) return ok();
  if (!a || !b || !output) return invalid_argument("pointer", "must not be null");
  return launched(launch_binary(kAdd, 0.f, a, b, output, size, thread_stream()), "add_f32");
}
extern "C" rtc_result rtc_mul_f32(const float* a, const float* b, float* output, size_t size) {
  RTC_OP_RANGE();
  if (size == 0) return ok();
  if (!a || !b || !output) return invalid_argument("pointer", "must not be null");
  return launched(launch_binary(kMul, 0.f, a, b, output, size, thread_stream()), "mul_f32");
}

// ------------------------------------------------------------------- softmax

extern "C" rtc_result rtc_softmax(const rtc_tensor* x, size_t dim, const rtc_tensor* out) {
  RTC_OP_RANGE();
  TRY(check_desc(x, "input"));
  TRY(check_desc(out, "out"));
  // activation.rs:93-105: float dtype first, then the dim range.
  if (!is_float(x->dtype)) return invalid_argument("dtype", "Softmax requires floating-point tensors");
  if (dim >= x->ndim) return invalid_dimension("softmax", dim, x->ndim - 1);
  TRY(check_output(x, out, "softmax"));
  TRY(require_f32(x, "softmax"));
  TRY(same_device(x, out, out));
  if (x->numel == 0) return ok();
  size_t outer, len, inner;
  split_dims(x, dim, &outer, &len, &inner);
  const bool last = dim + 1 == x->ndim;     // ndarray's minimum-stride axis
  if (on_host(x)) {
    // Units are outer slices ([len, inner] each): every lane stays whole.
    const size_t ub = len * inner * sizeof(float);
    const std::vector<size_t> iu{ub}, ou{ub};
    const std::vector<int> al{-1};
    return launched(staged_map({x->data}, iu, {out->data}, ou, al, outer,
                               staged_chunk_units(iu, ou, al),
                               [=](const void* const* din, void* const* dout, size_t, size_t cu,
                                   cudaStream_t s) {
                                 return launch_softmax((const float*)din[0], cu, len, inner,
                                                       last, (float*)dout[0], s);
                               }),
                    "softmax");
  }
  DeviceScope scope(x->device);
  if (!scope.ok()) return backend_error("cudaSetDevice", scope.error());
  return launched(launch_softmax(cf(x), outer, len, inner, last, f(out), thread_stream()),
                  "softmax");
}

// ---------------------------------------------------------- dim reductions

static rtc_result reduce_dim(DimReduce op, const rtc_tensor* x, size_t dim, const rtc_tensor* out,
                             const char* context) {
  TRY(check_desc(x, "input"));
  TRY(check_desc(out, "out"));
  // reduction.rs:76-82 / :112-118
  if (dim >= x->ndim) return invalid_dimension(context, dim, x->ndim - 1);
  size_t outer, len, inner;
  split_dims(x, dim, &outer, &len, &inner);
  const bool last = dim + 1 == x->ndim;     // ndarray's minimum-stride axis
  if (op != kDimSum && len == 0) return empty_tensor(context);
  if (out->numel != outer * inner || out->dtype != x->dtype)
    return shape_mismatch_vec(std::string(context) + " (output)", reduced_shape(x, dim),
                              shape_vec(out));
  TRY(require_f32(x, context));
  TRY(same_device(x, out, out));
  if (outer * inner == 0) return ok();
  if (on_host(x)) {
    const std::vector<size_t> iu{len * inner * sizeof(float)}, ou{inner * sizeof(float)};
    const std::vector<int> al{-1};
    return launched(staged_map({x->data}, iu, {out->data}, ou, al, outer,
                               staged_chunk_units(iu, ou, al),
                               [=](const void* const* din, void* const* dout, size_t, size_t cu,
                                   cudaStream_t s) {
                                 return launch_reduce_dim(op, (const float*)din[0], cu, len,
                                                          inner, last, (float*)dout[0], s);
                               }),
                    context);
  }
  DeviceScope scope(x->device);
  if (!scope.ok()) return backend_error("cudaSetDevice", scope.error());
  return launched(launch_reduce_dim(op, cf(x), outer, len, inner, last, f(out), thread_stream()),
                  context);
}

extern "C" rtc_result rtc_sum_dim(const rtc_tensor* x, size_t dim, const rtc_tensor* out) {
  RTC_OP_RANGE();
  return reduce_dim(kDimSum, x, dim, out, "sum_dim");
}
extern "C" rtc_result rtc_mean_dim(const rtc_tensor* x, size_t dim, const rtc_tensor* out) {
  RTC_OP_RANGE();
  return reduce_dim(kDimMean, x, dim, out, "mean_dim");
}
extern "C" rtc_result rtc_max_dim(const rtc_tensor* x, size_t dim, const rtc_tensor* out) {
  RTC_OP_RANGE();
  return reduce_dim(kDimMax, x, dim, out, "max_dim");
}

// ------------------------------------------------------- global reductions

static rtc_result global(const rtc_tensor* x, const char* op, bool empty_is_error, int want,
                         GlobalStats* st) {
  TRY(check_desc(x, "input"));
  if (x->numel == 0) {
    if (empty_is_error) return empty_tensor(op);
    st->sum = 0.0;
    return ok();
  }
  TRY(require_f32(x, op));
  if (on_host(x)) {
    std::vector<rtc_shard_summary> parts;
    cudaError_t e = staged_global_stats(cf(x), x->numel, &parts);
    if (e != cudaSuccess) return backend_error(op, e);
    double v[4];
    combine_summaries(parts.data(), parts.size(), v);
    st->sum = v[0];
    st->max = (float)v[2];
    st->min = (float)v[3];
    return ok();
  }
  if (x->device < 0) return invalid_argument("device", "invalid device ordinal");
  DeviceScope scope(x->device);
  if (!scope.ok()) return backend_error("cudaSetDevice", scope.error());
  cudaError_t e = exact_global_stats(cf(x), x->numel, x->device, want, thread_stream(), st);
  if (e != cudaSuccess) return backend_error(op, e);
  return ok();
}

extern "C" rtc_result rtc_sum(const rtc_tensor* x, double* out_value) {
  RTC_OP_RANGE();
  if (!out_value) return invalid_argument("out_value", "must not be null");
  GlobalStats st;
  TRY(global(x, "sum", false, kStatSum, &st));
  *out_value = st.sum;
  return ok();
}

extern "C" rtc_result rtc_mean(const rtc_tensor* x, double* out_value) {
  RTC_OP_RANGE();
  if (!out_value) return invalid_argument("out_value", "must not be null");
  GlobalStats st;
  TRY(global(x, "mean", true, kStatSum, &st));
  *out_value = st.sum / (double)x->numel;
  return ok();
}

extern "C" rtc_result rtc_max(const rtc_tensor* x, double* out_value) {
  RTC_OP_RANGE();
  if (!out_value) return invalid_argument("out_value", "must not be null");
  GlobalStats st;
  TRY(global(x, "max", true, kStatMax, &st));
  *out_value = (double)st.max;
  return ok();
}

extern "C" rtc_result rtc_min(const rtc_tensor* x, double* out_value) {
  RTC_OP_RANGE();
  if (!out_value) return invalid_argument("out_value", "must not be null");
  GlobalStats st;
  TRY(global(x, "min", true, kStatMin, &st));
  *out_value = (double)st.min;
  return ok();
}

extern "C" rtc_result rtc_sum_device(const rtc_tensor* x, double* device_out) {
  RTC_OP_RANGE();
  TRY(check_desc(x, "input"));
  if (!device_out) return invalid_argument("device_out", "must not be null");
  TRY(require_f32(x, "sum"));
  if (on_host(x) || x->device < 0)
    return invalid_argument("device", "rtc_sum_device needs a device tensor");
  DeviceScope scope(x->device);
  if (!scope.ok()) return backend_error("cudaSetDevice", scope.error());
  cudaStream_t s = thread_stream();
  if (x->numel == 0) return launched(cudaMemsetAsync(device_out, 0, sizeof(double), s), "sum");
  keep_pool_memory(x->device);
  const int nparts = stats_num_parts(x->device, x->numel);
  StatsPart* parts = nullptr;
  cudaError_t e = cudaMallocAsync(reinterpret_cast<void**>(&parts), nparts * sizeof(StatsPart), s);
  if (e != cudaSuccess) return backend_error("sum", e);
  e = launch_stats(cf(x), x->numel, parts, nparts, nullptr, s, device_out);
  cudaError_t e2 = cudaFreeAsync(parts, s);
  return launched(e != cudaSuccess ? e : e2, "sum");
}

extern "C" rtc_result rtc_stats(const rtc_tensor* x, double out[4]) {
  RTC_OP_RANGE();
  if (!out) return invalid_argument("out", "must not be null");
  GlobalStats st;
  TRY(global(x, "stats", true, kStatSum | kStatMax | kStatMin, &st));
  out[0] = st.sum;
  out[1] = st.sum / (double)x->numel;
  out[2] = (double)st.max;
  out[3] = (double)st.min;
  return ok();
}

// --------------------------------------------------- sharded reductions

extern "C" rtc_result rtc_shard_summary_local(const rtc_tensor* shard, rtc_shard_summary* out) {
  RTC_OP_RANGE();
  if (!out) return invalid_argument("out", "must not be null");
  TRY(check_desc(shard, "shard"));
  rtc_shard_summary s{};
  s.count = shard->numel;
  s.min_nonnan = INFINITY;
  if (shard->numel > 0 && on_host(shard)) {
    TRY(require_f32(shard, "shard_summary"));
    std::vector<rtc_shard_summary> parts;
    cudaError_t e = staged_global_stats(cf(shard), shard->numel, &parts);
    if (e != cudaSuccess) return backend_error("shard_summary", e);
    *out = compose_summaries(parts.data(), parts.size());
    return ok();
  }
  if (shard->numel > 0) {
    GlobalStats st;
    TRY(global(shard, "shard_summary", true, kStatSum | kStatMax | kStatMin, &st));
    s.sum = st.sum;
    s.max = st.max;
    s.max_kind = st.max_const ? 2 : 1;
    s.min_nonnan = st.min_nonnan;
    s.first_nan = st.first_nan ? 1 : 0;
  }
  *out = s;
  return ok();
}

// The reference folds max/min over the whole tensor in index order
// (reduction.rs:36-40, :58-62); composing the shards' summaries in shard
// order gives the same value.
// One process, several GPUs: the shards of each device are summarised by
// one host thread per device (so the devices work at once), then the
// summaries are folded in shard order.  Waits first for all work already queued on the shards'
// devices, since the shards may come from other streams.
extern "C" rtc_result rtc_sharded_stats(const rtc_tensor* shards, size_t n_shards,
                                        double out[4]) {
  RTC_OP_RANGE();
  if (!out) return invalid_argument("out", "must not be null");
  if (n_shards > 0 && !shards) return invalid_argument("shards", "must not be null");
  for (size_t i = 0; i < n_shards; i++) TRY(check_desc(&shards[i], "shard"));
  std::vector<int> devices;
  for (size_t i = 0; i < n_shards; i++)
    if (shards[i].device >= 0 &&
        std::find(devices.begin(), devices.end(), shards[i].device) == devices.end())
      devices.push_back(shards[i].device);
  for (int d : devices) {
    DeviceScope scope(d);
    if (!scope.ok()) return backend_error("cudaSetDevice", scope.error());
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return backend_error("cudaDeviceSynchronize", e);
  }
  // One worker per device (host-memory shards form their own group), each
  // summarising its shards in order.
  std::vector<rtc_shard_summary> parts(n_shards);
  std::vector<rtc_result> res(n_shards, ok());
  std::vector<std::vector<size_t>> groups;
  std::vector<int> group_device;
  for (size_t i = 0; i < n_shards; i++) {
    const int d = shards[i].device;
    size_t g = 0;
    while (g < group_device.size() && group_device[g] != d) g++;
    if (g == group_device.size()) {
      group_device.push_back(d);
      groups.emplace_back();
    }
    groups[g].push_back(i);
  }
  std::vector<std::thread> workers;
  workers.reserve(groups.size());
  for (const auto& idx : groups)
    workers.emplace_back([&, idx] {
      for (size_t i : idx) res[i] = rtc_shard_summary_local(&shards[i], &parts[i]);
    });
  for (auto& w : workers) w.join();
  rtc_result first_error = ok();
  for (size_t i = 0; i < n_shards; i++) {
    if (!res[i].success && first_error.success) first_error = res[i];
    else if (!res[i].success) std::free(res[i].error_msg);
  }
  if (!first_error.success) return first_error;
  return rtc_shard_combine(parts.data(), n_shards, out);
}

extern "C" rtc_result rtc_shard_combine(const rtc_shard_summary* parts, size_t n, double out[4]) {
  RTC_OP_RANGE();
  if (!out) return invalid_argument("out", "must not be null");
  if (n > 0 && !parts) return invalid_argument("parts", "must not be null");
  if (!combine_summaries(parts, n, out)) return empty_tensor("stats");
  return ok();
}

// ------------------------------------------------------------ broadcasting

// broadcast_shape (ops/broadcast.rs:32-53) and the plain op on the
// broadcast operands (:177-198).
static rtc_result broadcast_op(BinaryOp op, const rtc_tensor* a, const rtc_tensor* b,
                               const rtc_tensor* out, const char* context, bool float_only,
                               const char* float_reason) {
  TRY(check_desc(a, "a"));
  TRY(check_desc(b, "b"));
  TRY(check_desc(out, "out"));
  if (a->dtype != b->dtype)    // broadcast.rs:57-63 (Display form of the dtypes)
    return dtype_mismatch("broadcast_tensors", dtype_display(a->dtype), dtype_display(b->dtype));
  if (same_shape(a, b)) return binary(op, 0.f, a, b, out, context, float_only, float_reason);
  const size_t nd = a->ndim > b->ndim ? a->ndim : b->ndim;
  std::vector<size_t> os(nd), da(nd), db(nd);
  for (size_t i = 0; i < nd; i++) {
    da[i] = i < nd - a->ndim ? 1 : a->shape[i - (nd - a->ndim)];
    db[i] = i < nd - b->ndim ? 1 : b->shape[i - (nd - b->ndim)];
    if (da[i] != db[i] && da[i] != 1 && db[i] != 1)
      return fail(RTC_BROADCAST_ERROR, "Cannot broadcast shapes " + fmt_shape_pub(shape_vec(a)) +
                                           " and " + fmt_shape_pub(shape_vec(b)) +
                                           ": Incompatible shapes for broadcasting");
    os[i] = da[i] > db[i] ? da[i] : db[i];
  }
  if (float_only && !is_float(a->dtype)) return invalid_argument("dtype", float_reason);
  if (shape_vec(out) != os || out->dtype != a->dtype)
    return shape_mismatch_vec(std::string(context) + " (output)", os, shape_vec(out));
  TRY(require_f32(a, context));
  TRY(same_device(a, b, out));
  if (on_host(a)) return unsupported(std::string(context) + ": broadcast ops need device tensors");
  if (out->numel == 0) return ok();
  // Element strides (0 along broadcast dims), then merge dims that continue
  // each other in both operands.
  std::vector<long long> sh, as, bs;
  long long sa = 1, sb = 1;
  std::vector<long long> fa(nd), fb(nd);
  for (size_t i = nd; i-- > 0;) {
    fa[i] = da[i] == 1 ? 0 : sa;
    fb[i] = db[i] == 1 ? 0 : sb;
    sa *= (long long)da[i];
    sb *= (long long)db[i];
  }
  for (size_t i = 0; i < nd; i++) {
    if (os[i] == 1) continue;
    if (!sh.empty() && as.back() == fa[i] * (long long)os[i] &&
        bs.back() == fb[i] * (long long)os[i]) {
      sh.back() *= (long long)os[i];
      as.back() = fa[i];
      bs.back() = fb[i];
    } else {
      sh.push_back((long long)os[i]);
      as.push_back(fa[i]);
      bs.push_back(fb[i]);
    }
  }
  if (sh.empty()) {
    sh.push_back(1);
    as.push_back(0);
    bs.push_back(0);
  }
  if (sh.size() > (size_t)kMaxBcastDims)
    return unsupported(std::string(context) + ": more than 8 non-mergeable broadcast dims");
  BcastPlan plan{};
  plan.nd = (int)sh.size();
  for (int i = 0; i < plan.nd; i++) {
    plan.shape[i] = sh[i];
    plan.astride[i] = as[i];
    plan.bstride[i] = bs[i];
  }
  DeviceScope scope(a->device);
  if (!scope.ok()) return backend_error("cudaSetDevice", scope.error());
  return launched(launch_broadcast(op, cf(a), cf(b), f(out), out->numel, plan, thread_stream()),
                  context);
}

extern "C" rtc_result rtc_add_broadcast(const rtc_tensor* a, const rtc_tensor* b,
                                        const rtc_tensor* out) {
  RTC_OP_RANGE();
  return broadcast_op(kAdd, a, b, out, "element-wise addition", false, nullptr);
}
extern "C" rtc_result rtc_sub_broadcast(const rtc_tensor* a, const rtc_tensor* b,
                                        const rtc_tensor* out) {
  RTC_OP_RANGE();
  return broadcast_op(kSub, a, b, out, "element-wise subtraction", false, nullptr);
}
extern "C" rtc_result rtc_mul_broadcast(const rtc_tensor* a, const rtc_tensor* b,
                                        const rtc_tensor* out) {
  RTC_OP_RANGE();
  return broadcast_op(kMul, a, b, out, "element-wise multiplication", false, nullptr);
}
extern "C" rtc_result rtc_div_broadcast(const rtc_tensor* a, const rtc_tensor* b,
                                        const rtc_tensor* out) {
  RTC_OP_RANGE();
  return broadcast_op(kDiv, a, b, out, "element-wise division", true,
                      "Division requires floating-point tensors");
}

// ---------------------------------------------------------- nn optimizers

extern "C" rtc_result rtc_nn_adam_step(const rtc_tensor* p, const rtc_tensor* g,
                                       const rtc_tensor* m, const rtc_tensor* v, float lr,
                                       float beta1, float beta2, float eps, uint64_t t,
                                       const rtc_tensor* po, const rtc_tensor* mo,
                                       const rtc_tensor* vo) {
  RTC_OP_RANGE();
  TRY(check_desc(p, "params"));
  TRY(check_desc(g, "gradients"));
  TRY(check_desc(m, "m"));
  TRY(check_desc(v, "v"));
  TRY(check_desc(po, "params_out"));
  TRY(check_desc(mo, "m_out"));
  TRY(check_desc(vo, "v_out"));
  if (g->numel != p->numel) return shape_mismatch("Adam step", p, g);
  if (m->numel != p->numel) return shape_mismatch("Adam step", p, m);
  if (v->numel != p->numel) return shape_mismatch("Adam step", p, v);
  TRY(check_output(p, po, "Adam step"));
  if (mo->numel != p->numel) return shape_mismatch("Adam step (output)", p, mo);
  if (vo->numel != p->numel) return shape_mismatch("Adam step (output)", p, vo);
  TRY(require_f32(p, "Adam step"));
  TRY(require_f32(g, "Adam step"));
  TRY(require_f32(m, "Adam step"));
  TRY(require_f32(v, "Adam step"));
  TRY(same_device(p, g, m));
  TRY(same_device(p, v, po));
  TRY(same_device(p, mo, vo));
  if (p->numel == 0) return ok();
  // nn/optim.rs:264-268: t as f32, bias corrections with f32 powf.
  const float tf = (float)t;
  NnAdamCoeffs c;
  c.b1 = beta1;
  c.one_minus_b1 = 1.0f - beta1;
  c.b2 = beta2;
  c.one_minus_b2 = 1.0f - beta2;
  c.bc1 = 1.0f - powf(beta1, tf);
  c.bc2 = 1.0f - powf(beta2, tf);
  c.lr = lr;
  c.eps = eps;
  if (on_host(p)) {
    const std::vector<size_t> iu{4, 4, 4, 4}, ou{4, 4, 4};
    const std::vector<int> al{0, 2, 3};
    return launched(staged_map({p->data, g->data, m->data, v->data}, iu,
                               {po->data, mo->data, vo->data}, ou, al, p->numel,
                               staged_chunk_units(iu, ou, al),
                               [=](const void* const* din, void* const* dout, size_t, size_t cu,
                                   cudaStream_t s) {
                                 return launch_nn_adam((const float*)din[0], (const float*)din[1],
                                                       (const float*)din[2], (const float*)din[3],
                                                       (float*)dout[0], (float*)dout[1],
                                                       (float*)dout[2], cu, c, s);
                               }),
                    "Adam step");
  }
  DeviceScope scope(p->device);
  if (!scope.ok()) return backend_error("cudaSetDevice", scope.error());
  return launched(launch_nn_adam(cf(p), cf(g), cf(m), cf(v), f(po), f(mo), f(vo), p->numel, c,
                                 thread_stream()),
                  "Adam step");
}

extern "C" rtc_result rtc_nn_sgd_step(const rtc_tensor* p, const rtc_tensor* g,
                                      const rtc_tensor* vel, float lr, float momentum,
                                      float weight_decay, const rtc_tensor* po,
                                      const rtc_tensor* vo) {
  RTC_OP_RANGE();
  TRY(check_desc(p, "params"));
  TRY(check_desc(g, "gradients"));
  TRY(check_desc(po, "params_out"));
  // nn/optim.rs:160-166 compares element counts.
  if (p->numel != g->numel) return shape_mismatch("SGD step", p, g);
  const bool mom = momentum > 0.0f;
  if (mom) {
    TRY(check_desc(vel, "velocity"));
    TRY(check_desc(vo, "velocity_out"));
    if (vel->numel != p->numel) return shape_mismatch("SGD step", p, vel);
    if (vo->numel != p->numel) return shape_mismatch("SGD step (output)", p, vo);
    TRY(require_f32(vel, "SGD step"));
  }
  TRY(check_output(p, po, "SGD step"));
  TRY(require_f32(p, "SGD step"));
  TRY(require_f32(g, "SGD step"));
  TRY(same_device(p, g, po));
  if (mom) TRY(same_device(p, vel, vo));
  if (p->numel == 0) return ok();
  if (on_host(p)) {
    if (mom) {
      const std::vector<size_t> iu{4, 4, 4}, ou{4, 4};
      const std::vector<int> al{0, 2};
      return launched(staged_map({p->data, g->data, vel->data}, iu, {po->data, vo->data}, ou, al,
                                 p->numel, staged_chunk_units(iu, ou, al),
                                 [=](const void* const* din, void* const* dout, size_t,
                                     size_t cu, cudaStream_t s) {
                                   return launch_nn_sgd((const float*)din[0],
                                                        (const float*)din[1],
                                                        (const float*)din[2], (float*)dout[0],
                                                        (float*)dout[1], cu, lr, momentum,
                                                        weight_decay, s);
                                 }),
                      "SGD step");
    }
    const std::vector<size_t> iu{4, 4}, ou{4};
    const std::vector<int> al{0};
    return launched(staged_map({p->data, g->data}, iu, {po->data}, ou, al, p->numel,
                               staged_chunk_units(iu, ou, al),
                               [=](const void* const* din, void* const* dout, size_t, size_t cu,
                                   cudaStream_t s) {
                                 return launch_nn_sgd((const float*)din[0], (const float*)din[1],
                                                      nullptr, (float*)dout[0], nullptr, cu, lr,
                                                      momentum, weight_decay, s);
                               }),
                    "SGD step");
  }
  DeviceScope scope(p->device);
  if (!scope.ok()) return backend_error("cudaSetDevice", scope.error());
  return launched(launch_nn_sgd(cf(p), cf(g), mom ? cf(vel) : nullptr, f(po),
                                mom ? f(vo) : nullptr, p->numel, lr, momentum, weight_decay,
                                thread_stream()),
                  "SGD step");
}

// ------------------------------------------------------------- optimizers

// optimizer.rs:242-271, in order.  NaN passes (the comparisons are false).
static rtc_result adam_hyper_checks(double lr, double b1, double b2, double eps, uint64_t t) {
  if (lr <= 0.0) return invalid_argument("learning_rate", "must be positive, got " + rust_f64(lr));
  if (b1 <= 0.0 || b1 >= 1.0) return invalid_argument("beta1", "must be in (0, 1), got " + rust_f64(b1));
  if (b2 <= 0.0 || b2 >= 1.0) return invalid_argument("beta2", "must be in (0, 1), got " + rust_f64(b2));
  if (eps <= 0.0) return invalid_argument("epsilon", "must be positive, got " + rust_f64(eps));
  if (t == 0) return invalid_argument("timestep", "must be >= 1");
  return ok();
}

static rtc_result adam_common(const rtc_tensor* p, const rtc_tensor* g, const rtc_tensor* m,
                              const rtc_tensor* v, double lr, double b1, double b2, double eps,
                              double wd, uint64_t t, const rtc_tensor* po, const rtc_tensor* mo,
                              const rtc_tensor* vo, bool adamw) {
  TRY(check_desc(p, "params"));
  TRY(check_desc(g, "gradients"));
  TRY(check_desc(m, "m"));
  TRY(check_desc(v, "v"));
  TRY(check_desc(po, "params_out"));
  TRY(check_desc(mo, "m_out"));
  TRY(check_desc(vo, "v_out"));
  // optimizer.rs:392-397: adamw rejects a negative weight decay first.
  if (adamw && wd < 0.0)
    return invalid_argument("weight_decay", "must be non-negative, got " + rust_f64(wd));
  // optimizer.rs:219-239
  if (!same_shape(p, g)) return shape_mismatch("adam_update (params vs gradients)", p, g);
  if (!same_shape(p, m)) return shape_mismatch("adam_update (params vs m)", p, m);
  if (!same_shape(p, v)) return shape_mismatch("adam_update (params vs v)", p, v);
  TRY(adam_hyper_checks(lr, b1, b2, eps, t));
  // optimizer.rs:284-345: all f32 or all f64, else DTypeMismatch.
  const bool all_f32 = p->dtype == RTC_F32 && g->dtype == RTC_F32 && m->dtype == RTC_F32 &&
                       v->dtype == RTC_F32;
  const bool all_f64 = p->dtype == RTC_F64 && g->dtype == RTC_F64 && m->dtype == RTC_F64 &&
                       v->dtype == RTC_F64;
  if (!all_f32 && !all_f64)
    return dtype_mismatch("adam_update (only floating-point supported)", "float32 or float64",
                          dtype_display(p->dtype));
  TRY(check_output(p, po, "adam_update"));
  TRY(check_output(p, mo, "adam_update"));
  TRY(check_output(p, vo, "adam_update"));
  TRY(require_f32(p, "adam_update"));
  TRY(same_device(p, g, m));
  TRY(same_device(p, v, po));
  TRY(same_device(p, mo, vo));
  if (p->numel == 0) return ok();
  // Host-side coefficients, rounded as optimizer.rs:278-309 and :413-418 do.
  const double td = (double)t;
  const double bc1 = 1.0 - std::pow(b1, td);
  const double bc2 = 1.0 - std::pow(b2, td);
  AdamCoeffs c;
  c.b1 = (float)b1;
  c.one_minus_b1 = 1.0f - c.b1;
  c.b2 = (float)b2;
  c.one_minus_b2 = 1.0f - c.b2;
  c.bc1 = (float)bc1;
  c.bc2 = (float)bc2;
  c.eps = (float)eps;
  c.lr = (float)lr;
  c.decay = adamw && wd > 0.0;
  c.lr_wd = (float)(lr * wd);
  if (on_host(p)) {
    const std::vector<size_t> iu{4, 4, 4, 4}, ou{4, 4, 4};
    const std::vector<int> al{0, 2, 3};   // p', m', v' overwrite p, m, v on the device
    return launched(staged_map({p->data, g->data, m->data, v->data}, iu,
                               {po->data, mo->data, vo->data}, ou, al, p->numel,
                               staged_chunk_units(iu, ou, al),
                               [=](const void* const* din, void* const* dout, size_t, size_t cu,
                                   cudaStream_t s) {
                                 return launch_adam((const float*)din[0], (const float*)din[1],
                                                    (const float*)din[2], (const float*)din[3],
                                                    (float*)dout[0], (float*)dout[1],
                                                    (float*)dout[2], cu, c, s);
                               }),
                    adamw ? "adamw_update" : "adam_update");
  }
  DeviceScope scope(p->device);
  if (!scope.ok()) return backend_error("cudaSetDevice", scope.error());
  return launched(launch_adam(cf(p), cf(g), cf(m), cf(v), f(po), f(mo), f(vo), p->numel, c,
                              thread_stream()),
                  adamw ? "adamw_update" : "adam_update");
}

extern "C" rtc_result rtc_adam_update(const rtc_tensor* params, const rtc_tensor* grads,
                                      const rtc_tensor* m, const rtc_tensor* v,
                                      double learning_rate, double beta1, double beta2,
                                      double epsilon, uint64_t timestep,
                                      const rtc_tensor* params_out, const rtc_tensor* m_out,
                                      const rtc_tensor* v_out) {
  RTC_OP_RANGE();
  return adam_common(params, grads, m, v, learning_rate, beta1, beta2, epsilon, 0.0, timestep,
                     params_out, m_out, v_out, false);
}

extern "C" rtc_result rtc_adamw_update(const rtc_tensor* params, const rtc_tensor* grads,
                                       const rtc_tensor* m, const rtc_tensor* v,
                                       double learning_rate, double beta1, double beta2,
                                       double epsilon, double weight_decay, uint64_t timestep,
                                       const rtc_tensor* params_out, const rtc_tensor* m_out,
                                       const rtc_tensor* v_out) {
  RTC_OP_RANGE();
  return adam_common(params, grads, m, v, learning_rate, beta1, beta2, epsilon, weight_decay,
                     timestep, params_out, m_out, v_out, true);
}

// optimizer.rs:42-86: shape, dtype, learning rate; float only.
extern "C" rtc_result rtc_sgd_update(const rtc_tensor* p, const rtc_tensor* g, double lr,
                                     const rtc_tensor* po) {
  RTC_OP_RANGE();
  TRY(check_desc(p, "params"));
  TRY(check_desc(g, "gradients"));
  TRY(check_desc(po, "params_out"));
  if (!same_shape(p, g)) return shape_mismatch("sgd_update", p, g);
  if (p->dtype != g->dtype)
    return dtype_mismatch("sgd_update", dtype_display(p->dtype), dtype_display(g->dtype));
  if (lr <= 0.0) return invalid_argument("learning_rate", "must be positive, got " + rust_f64(lr));
  if (!is_float(p->dtype))
    return dtype_mismatch("sgd_update (only floating-point supported)", "float32 or float64",
                          dtype_display(p->dtype));
  TRY(check_output(p, po, "sgd_update"));
  TRY(require_f32(p, "sgd_update"));
  TRY(same_device(p, g, po));
  if (p->numel == 0) return ok();
  if (on_host(p)) {
    const std::vector<size_t> iu{4, 4}, ou{4};
    const std::vector<int> al{0};
    const float flr = (float)lr;
    return launched(staged_map({p->data, g->data}, iu, {po->data}, ou, al, p->numel,
                               staged_chunk_units(iu, ou, al),
                               [=](const void* const* din, void* const* dout, size_t, size_t cu,
                                   cudaStream_t s) {
                                 return launch_sgd((const float*)din[0], (const float*)din[1],
                                                   (float*)dout[0], cu, flr, s);
                               }),
                    "sgd_update");
  }
  DeviceScope scope(p->device);
  if (!scope.ok()) return backend_error("cudaSetDevice", scope.error());
  return launched(launch_sgd(cf(p), cf(g), f(po), p->numel, (float)lr, thread_stream()),
                  "sgd_update");
}

// optimizer.rs:108-177: shapes, learning rate, momentum in [0, 1), dtypes.
extern "C" rtc_result rtc_sgd_momentum_update(const rtc_tensor* p, const rtc_tensor* g,
                                              const rtc_tensor* vel, double lr, double momentum,
                                              const rtc_tensor* po, const rtc_tensor* vo) {
  RTC_OP_RANGE();
  TRY(check_desc(p, "params"));
  TRY(check_desc(g, "gradients"));
  TRY(check_desc(vel, "velocity"));
  TRY(check_desc(po, "params_out"));
  TRY(check_desc(vo, "velocity_out"));
  if (!same_shape(p, g)) return shape_mismatch("sgd_momentum_update (params vs gradients)", p, g);
  if (!same_shape(p, vel)) return shape_mismatch("sgd_momentum_update (params vs velocity)", p, vel);
  if (lr <= 0.0) return invalid_argument("learning_rate", "must be positive, got " + rust_f64(lr));
  if (!(momentum >= 0.0 && momentum < 1.0))
    return invalid_argument("momentum", "must be in [0, 1), got " + rust_f64(momentum));
  const bool all_f32 = p->dtype == RTC_F32 && g->dtype == RTC_F32 && vel->dtype == RTC_F32;
  const bool all_f64 = p->dtype == RTC_F64 && g->dtype == RTC_F64 && vel->dtype == RTC_F64;
  if (!all_f32 && !all_f64)
    return dtype_mismatch("sgd_momentum_update (only floating-point supported)",
                          "float32 or float64", dtype_display(p->dtype));
  TRY(check_output(p, po, "sgd_momentum_update"));
  TRY(check_output(p, vo, "sgd_momentum_update"));
  TRY(require_f32(p, "sgd_momentum_update"));
  TRY(same_device(p, g, vel));
  TRY(same_device(p, po, vo));
  if (p->numel == 0) return ok();
  if (on_host(p)) {
    const std::vector<size_t> iu{4, 4, 4}, ou{4, 4};
    const std::vector<int> al{0, 2};
    const float flr = (float)lr, fm = (float)momentum;
    return launched(staged_map({p->data, g->data, vel->data}, iu, {po->data, vo->data}, ou, al,
                               p->numel, staged_chunk_units(iu, ou, al),
                               [=](const void* const* din, void* const* dout, size_t, size_t cu,
                                   cudaStream_t s) {
                                 return launch_sgd_momentum(
                                     (const float*)din[0], (const float*)din[1],
                                     (const float*)din[2], (float*)dout[0], (float*)dout[1], cu,
                                     flr, fm, s);
                               }),
                    "sgd_momentum_update");
  }
  DeviceScope scope(p->device);
  if (!scope.ok()) return backend_error("cudaSetDevice", scope.error());
  return launched(launch_sgd_momentum(cf(p), cf(g), cf(vel), f(po), f(vo), p->numel, (float)lr,
                                      (float)momentum, thread_stream()),
                  "sgd_momentum_update");
}
