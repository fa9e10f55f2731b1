// abi_backward.cu — C-ABI entry points for autograd's gradient functions
// (rusttorch-core src/autograd/ops.rs, GradFn::backward).
//
// The reference has no C entry point for these: its autograd runs each
// backward as ops::* calls on the CPU.  Each function here produces the same
// tensors from one fused kernel.  A NULL gradient output stands for the
// reference's `None` (that input does not require grad).  Argument errors
// are those of the ops::* call that would fail first in the reference.
#include "rt_abi_util.h"
#include "rt_staging.h"

using namespace rt;

namespace {

bool on_host(const rtc_tensor* t) { return t->device == RTC_HOST_MEMORY; }

const char* kMulCtx = "element-wise multiplication";
const char* kDivCtx = "element-wise division";

// ops::mul / ops::div argument checks: dtype first, then shape
// (ops/elementwise.rs:15-28, :163-183).
rtc_result pair(const rtc_tensor* x, const rtc_tensor* y, const char* context, bool div) {
  if (x->dtype != y->dtype)
    return dtype_mismatch(context, dtype_debug(x->dtype), dtype_debug(y->dtype));
  if (!same_shape(x, y)) return shape_mismatch(context, x, y);
  if (div && !is_float(x->dtype))
    return invalid_argument("dtype", "Division requires floating-point tensors");
  return ok();
}

// Streams host tensors through the GPU, or launches on the device.
template <class Launch>
rtc_result run(const std::vector<const rtc_tensor*>& ins, const std::vector<const rtc_tensor*>& outs,
               size_t n, const char* context, Launch launch) {
  if (n == 0) return ok();
  const rtc_tensor* first = ins[0];
  if (on_host(first)) {
    std::vector<const void*> hin;
    std::vector<void*> hout;
    for (auto* t : ins) hin.push_back(t->data);
    for (auto* t : outs) hout.push_back(t->data);
    const std::vector<size_t> iu(ins.size(), 4), ou(outs.size(), 4);
    const std::vector<int> al(outs.size(), -1);
    return launched(staged_map(hin, iu, hout, ou, al, n, staged_chunk_units(iu, ou, al),
                               [=](const void* const* din, void* const* dout, size_t,
                                   size_t cu, cudaStream_t s) {
                                 return launch(din, dout, cu, s);
                               }),
                    context);
  }
  DeviceScope scope(first->device);
  if (!scope.ok()) return backend_error("cudaSetDevice", scope.error());
  std::vector<const void*> din;
  std::vector<void*> dout;
  for (auto* t : ins) din.push_back(t->data);
  for (auto* t : outs) dout.push_back(t->data);
  return launched(launch(din.data(), dout.data(), n, thread_stream()), context);
}

rtc_result all_same_device(const std::vector<const rtc_tensor*>& ts) {
  for (size_t i = 1; i < ts.size(); i++) TRY(same_device(ts[0], ts[i], ts[i]));
  return ok();
}

// relu / sigmoid / tanh: grad = mul(grad_output, h(saved)).
rtc_result grad_unary(GradUnaryOp op, const rtc_tensor* g, const rtc_tensor* saved,
                      const rtc_tensor* out, const char* name) {
  TRY(check_desc(g, "grad_output"));
  TRY(check_desc(saved, name));
  TRY(check_desc(out, "grad_input"));
  TRY(pair(g, saved, kMulCtx, false));
  TRY(check_output(g, out, kMulCtx));
  TRY(require_f32(g, kMulCtx));
  TRY(same_device(g, saved, out));
  return run({g, saved}, {out}, g->numel, kMulCtx,
             [=](const void* const* din, void* const* dout, size_t n, cudaStream_t s) {
               return launch_grad_unary(op, (const float*)din[0], (const float*)din[1],
                                        (float*)dout[0], n, s);
             });
}

}  // namespace

extern "C" rtc_result rtc_relu_backward(const rtc_tensor* grad_output, const rtc_tensor* input,
                                        const rtc_tensor* grad_input) {
  RTC_OP_RANGE();
  return grad_unary(kGradRelu, grad_output, input, grad_input, "input");
}

extern "C" rtc_result rtc_sigmoid_backward(const rtc_tensor* grad_output,
                                           const rtc_tensor* output,
                                           const rtc_tensor* grad_input) {
  RTC_OP_RANGE();
  return grad_unary(kGradSigmoid, grad_output, output, grad_input, "output");
}

extern "C" rtc_result rtc_tanh_backward(const rtc_tensor* grad_output, const rtc_tensor* output,
                                        const rtc_tensor* grad_input) {
  RTC_OP_RANGE();
  return grad_unary(kGradTanh, grad_output, output, grad_input, "output");
}

// GeluBackward (ops.rs:3102-3125) walks input_saved's elements and indexes
// grad_output by position; the result has the input's shape.
extern "C" rtc_result rtc_gelu_backward(const rtc_tensor* grad_output, const rtc_tensor* input,
                                        const rtc_tensor* grad_input) {
  RTC_OP_RANGE();
  const char* context = "gelu backward";
  TRY(check_desc(grad_output, "grad_output"));
  TRY(check_desc(input, "input"));
  TRY(check_desc(grad_input, "grad_input"));
  if (grad_output->numel != input->numel) return shape_mismatch(context, input, grad_output);
  TRY(check_output(input, grad_input, context));
  TRY(require_f32(input, context));
  TRY(require_f32(grad_output, context));
  TRY(same_device(grad_output, input, grad_input));
  return run({grad_output, input}, {grad_input}, input->numel, context,
             [](const void* const* din, void* const* dout, size_t n, cudaStream_t s) {
               return launch_grad_unary(kGradGelu, (const float*)din[0], (const float*)din[1],
                                        (float*)dout[0], n, s);
             });
}

// gelu_forward (ops.rs:3131-3141): autograd's own GELU, whose cubic term is
// ((0.044715*x)*x)*x rather than ops::gelu's 0.044715*((x*x)*x).
extern "C" rtc_result rtc_autograd_gelu(const rtc_tensor* input, const rtc_tensor* output) {
  RTC_OP_RANGE();
  const char* context = "gelu_forward";
  TRY(check_desc(input, "input"));
  TRY(check_desc(output, "output"));
  TRY(check_output(input, output, context));
  TRY(require_f32(input, context));
  TRY(same_device(input, output, output));
  return run({input}, {output}, input->numel, context,
             [](const void* const* din, void* const* dout, size_t n, cudaStream_t s) {
               return launch_gelu_autograd((const float*)din[0], (float*)dout[0], n, s);
             });
}

// AddBackward / SubBackward (ops.rs:133-149, :175-192): clones of
// grad_output, negated for SubBackward's b.
static rtc_result add_sub_backward(GradBinaryOp op, const rtc_tensor* g, const rtc_tensor* ga,
                                   const rtc_tensor* gb, const char* context) {
  TRY(check_desc(g, "grad_output"));
  if (ga) TRY(check_desc(ga, "grad_a"));
  if (gb) TRY(check_desc(gb, "grad_b"));
  if (ga) TRY(check_output(g, ga, context));
  if (gb) TRY(check_output(g, gb, context));
  TRY(require_f32(g, context));
  std::vector<const rtc_tensor*> outs;
  if (ga) outs.push_back(ga);
  if (gb) outs.push_back(gb);
  if (outs.empty()) return ok();
  std::vector<const rtc_tensor*> all{g};
  all.insert(all.end(), outs.begin(), outs.end());
  TRY(all_same_device(all));
  const bool has_a = ga != nullptr, has_b = gb != nullptr;
  return run({g}, outs, g->numel, context,
             [=](const void* const* din, void* const* dout, size_t n, cudaStream_t s) {
               float* oa = has_a ? (float*)dout[0] : nullptr;
               float* ob = has_b ? (float*)dout[has_a ? 1 : 0] : nullptr;
               return launch_grad_binary(op, (const float*)din[0], nullptr, nullptr, oa, ob, n,
                                         s);
             });
}

extern "C" rtc_result rtc_add_backward(const rtc_tensor* grad_output, const rtc_tensor* grad_a,
                                       const rtc_tensor* grad_b) {
  RTC_OP_RANGE();
  return add_sub_backward(kGradAdd, grad_output, grad_a, grad_b, "add backward");
}

extern "C" rtc_result rtc_sub_backward(const rtc_tensor* grad_output, const rtc_tensor* grad_a,
                                       const rtc_tensor* grad_b) {
  RTC_OP_RANGE();
  return add_sub_backward(kGradSub, grad_output, grad_a, grad_b, "sub backward");
}

// MulBackward (ops.rs:219-236): grad_a = g*b, grad_b = g*a.
// DivBackward (ops.rs:267-290): grad_a = g/b, grad_b = g * ((-a) / (b*b)).
static rtc_result mul_div_backward(GradBinaryOp op, const rtc_tensor* g, const rtc_tensor* a,
                                   const rtc_tensor* b, const rtc_tensor* ga,
                                   const rtc_tensor* gb) {
  const bool div = op == kGradDiv;
  const char* first = div ? kDivCtx : kMulCtx;
  TRY(check_desc(g, "grad_output"));
  TRY(check_desc(a, "a"));
  TRY(check_desc(b, "b"));
  if (ga) TRY(check_desc(ga, "grad_a"));
  if (gb) TRY(check_desc(gb, "grad_b"));
  if (ga) {
    TRY(pair(g, b, first, div));
    TRY(check_output(g, ga, first));
  }
  if (gb) {
    if (div) TRY(pair(a, b, kDivCtx, true));   // (-a) / (b*b)
    TRY(pair(g, a, kMulCtx, false));
    TRY(check_output(g, gb, kMulCtx));
  }
  if (!ga && !gb) return ok();
  TRY(require_f32(g, first));
  // Operands each launch reads: mul needs b for grad_a and a for grad_b;
  // div's grad_b needs both.
  const bool need_a = gb != nullptr;
  const bool need_b = ga != nullptr || div;
  std::vector<const rtc_tensor*> ins{g}, outs, all{g};
  if (need_a) ins.push_back(a);
  if (need_b) ins.push_back(b);
  if (ga) outs.push_back(ga);
  if (gb) outs.push_back(gb);
  all.insert(all.end(), ins.begin() + 1, ins.end());
  all.insert(all.end(), outs.begin(), outs.end());
  TRY(all_same_device(all));
  const bool has_a = ga != nullptr, has_b = gb != nullptr;
  return run(ins, outs, g->numel, first,
             [=](const void* const* din, void* const* dout, size_t n, cudaStream_t s) {
               const float* pa = need_a ? (const float*)din[1] : nullptr;
               const float* pb = need_b ? (const float*)din[need_a ? 2 : 1] : nullptr;
               float* oa = has_a ? (float*)dout[0] : nullptr;
               float* ob = has_b ? (float*)dout[has_a ? 1 : 0] : nullptr;
               return launch_grad_binary(op, (const float*)din[0], pa, pb, oa, ob, n, s);
             });
}

extern "C" rtc_result rtc_mul_backward(const rtc_tensor* grad_output, const rtc_tensor* a,
                                       const rtc_tensor* b, const rtc_tensor* grad_a,
                                       const rtc_tensor* grad_b) {
  RTC_OP_RANGE();
  return mul_div_backward(kGradMul, grad_output, a, b, grad_a, grad_b);
}

extern "C" rtc_result rtc_div_backward(const rtc_tensor* grad_output, const rtc_tensor* a,
                                       const rtc_tensor* b, const rtc_tensor* grad_a,
                                       const rtc_tensor* grad_b) {
  RTC_OP_RANGE();
  return mul_div_backward(kGradDiv, grad_output, a, b, grad_a, grad_b);
}

// SumBackward / MeanBackward (ops.rs:501-511, :542-552): grad_output.item()
// (one element, else InvalidArgument), then Tensor::full(input shape, v).
// The value is read on the device, so no host round trip.
static rtc_result fill_backward(const rtc_tensor* g, const rtc_tensor* gi, bool mean,
                                const char* context) {
  TRY(check_desc(g, "grad_output"));
  TRY(check_desc(gi, "grad_input"));
  if (g->numel != 1)
    return invalid_argument("tensor", "item() requires a single-element tensor, got " +
                                          std::to_string(g->numel) + " elements");
  TRY(require_f32(g, context));
  TRY(require_f32(gi, context));
  if (on_host(g) || on_host(gi))
    return invalid_argument("device", std::string(context) + " needs device tensors");
  TRY(same_device(g, gi, gi));
  if (gi->numel == 0) return ok();
  DeviceScope scope(gi->device);
  if (!scope.ok()) return backend_error("cudaSetDevice", scope.error());
  return launched(launch_fill_from(cf(g), f(gi), gi->numel, (double)gi->numel, mean,
                                   thread_stream()),
                  context);
}

extern "C" rtc_result rtc_sum_backward(const rtc_tensor* grad_output,
                                       const rtc_tensor* grad_input) {
  RTC_OP_RANGE();
  return fill_backward(grad_output, grad_input, false, "sum backward");
}

extern "C" rtc_result rtc_mean_backward(const rtc_tensor* grad_output,
                                        const rtc_tensor* grad_input) {
  RTC_OP_RANGE();
  return fill_backward(grad_output, grad_input, true, "mean backward");
}

// BroadcastAddBackward's reduce_to_shape (ops.rs:627-681) for one operand:
// grad (the output's shape) folded back to `orig`'s shape, in the
// reference's order:
//   same shape                 -> copy
//   2-D [1, C] from [R, C]     -> column sums, rows in order from 0.0
//   2-D [R, 1] from [R, C]     -> row sums, one chain per row from 0.0
//   same element count         -> copy (a reshape)
//   otherwise                  -> result[i % m] += grad[i] for i in order
static rtc_result reduce_to_shape(const rtc_tensor* g, const rtc_tensor* o, cudaStream_t s) {
  const size_t len = g->numel, m = o->numel;
  const float* x = cf(g);
  float* out = f(o);
  const char* ctx = "broadcast_add backward";
  auto copy = [&]() {
    return launched(len ? cudaMemcpyAsync(out, x, len * sizeof(float), cudaMemcpyDeviceToDevice, s)
                        : cudaSuccess,
                    ctx);
  };
  if (same_shape(g, o)) return copy();
  if (g->ndim == 2 && o->ndim == 2) {
    const size_t R = g->shape[0], C = g->shape[1];
    if (o->shape[0] == 1 && o->shape[1] == C)
      return launched(launch_reduce_dim(kDimSum, x, 1, R, C, false, out, s), ctx);
    if (o->shape[1] == 1 && o->shape[0] == R)
      return launched(launch_lane_chain_sum(x, R, C, out, s), ctx);
  }
  if (len == m) return copy();
  if (m == 0) return invalid_argument("grad", "cannot fold a gradient onto an empty shape");
  const size_t blocks = len / m, rem = len % m;
  cudaError_t e;
  if (blocks == 0) {
    e = cudaMemsetAsync(out, 0, m * sizeof(float), s);
  } else if (m == 1) {
    e = launch_lane_chain_sum(x, 1, blocks, out, s);
  } else {
    e = launch_reduce_dim(kDimSum, x, 1, blocks, m, false, out, s);
  }
  // the ragged last block: out[j] += grad[blocks*m + j] for j < rem
  if (e == cudaSuccess && rem)
    e = launch_binary(kAdd, 0.0f, out, x + blocks * m, out, rem, s);
  return launched(e, ctx);
}

extern "C" rtc_result rtc_broadcast_add_backward(const rtc_tensor* grad_output,
                                                 const rtc_tensor* grad_a,
                                                 const rtc_tensor* grad_b) {
  RTC_OP_RANGE();
  const char* context = "broadcast_add backward";
  TRY(check_desc(grad_output, "grad_output"));
  if (grad_a) TRY(check_desc(grad_a, "grad_a"));
  if (grad_b) TRY(check_desc(grad_b, "grad_b"));
  TRY(require_f32(grad_output, context));
  if (grad_a) TRY(require_f32(grad_a, context));
  if (grad_b) TRY(require_f32(grad_b, context));
  for (const rtc_tensor* t : {grad_output, grad_a, grad_b})
    if (t && on_host(t))
      return invalid_argument("device", "broadcast_add backward needs device tensors");
  if (grad_a) TRY(same_device(grad_output, grad_a, grad_a));
  if (grad_b) TRY(same_device(grad_output, grad_b, grad_b));
  if (!grad_a && !grad_b) return ok();
  DeviceScope scope(grad_output->device);
  if (!scope.ok()) return backend_error("cudaSetDevice", scope.error());
  cudaStream_t s = thread_stream();
  if (grad_a) TRY(reduce_to_shape(grad_output, grad_a, s));
  if (grad_b) TRY(reduce_to_shape(grad_output, grad_b, s));
  return ok();
}
