// backward.cu — the elementwise gradient functions of rusttorch-core's
// autograd (src/autograd/ops.rs, GradFn::backward), one fused kernel each.
//
// The reference builds every gradient from ops::* calls (a mask tensor, a
// ones tensor, then sub and mul), each a separate pass that allocates.  Here
// each backward reads its saved tensors and grad_output once and writes the
// gradients once, with the reference's f32 operations in the reference's
// order, so results are bit-identical: 12 B per element for one-input
// backwards, 20 B for mul/div with both gradients.
#include "rt_internal.h"
#include "rt_map.cuh"
#include "rt_ops.cuh"

namespace rt {
namespace {

// ops.rs:380-387: mask = x > 0 ? 1 : 0 (NaN -> 0); grad = grad_output * mask
struct GradRelu {
  RT_HD float operator()(float g, float x) const { return fmul(g, x > 0.0f ? 1.0f : 0.0f); }
};
// ops.rs:424-427: grad = grad_output * (y * (1 - y)), y = sigmoid(x) saved
struct GradSigmoid {
  RT_HD float operator()(float g, float y) const { return fmul(g, fmul(y, fsub(1.0f, y))); }
};
// ops.rs:465-468: grad = grad_output * (1 - y*y), y = tanh(x) saved
struct GradTanh {
  RT_HD float operator()(float g, float y) const { return fmul(g, fsub(1.0f, fmul(y, y))); }
};
// ops.rs:3110-3118, with k = sqrt(2/pi) in f32 and c3 = 3 * 0.044715 in f32:
//   inner = k * (x + 0.044715*((x*x)*x));  t = tanh(inner);  sech2 = 1 - t*t
//   d_inner = k * (1 + (c3*x)*x)
//   grad = g * (0.5*(1 + t) + ((0.5*x)*sech2)*d_inner)
struct GradGelu {
  static constexpr bool kHeavy = true;   // one vector per thread, 64 blocks/SM: 0.48 vs 0.44
  float k, c3;
  RT_HD float operator()(float g, float x) const {
    const float x3 = fmul(fmul(x, x), x);
    const float inner = fmul(k, fadd(x, fmul(0.044715f, x3)));
    const float t = tanhf_glibc(inner);
    const float sech2 = fsub(1.0f, fmul(t, t));
    const float d_inner = fmul(k, fadd(1.0f, fmul(fmul(c3, x), x)));
    const float a = fmul(0.5f, fadd(1.0f, t));
    const float b = fmul(fmul(fmul(0.5f, x), sech2), d_inner);
    return fmul(g, fadd(a, b));
  }
};
// ops.rs:3136-3141 (autograd gelu_forward, not ops::gelu):
//   (0.5*x) * (1 + tanh(k * (x + ((0.044715*x)*x)*x)))
struct OpGeluAutograd {
  static constexpr bool kHeavy = true;
  float k;
  RT_HD float operator()(float x) const {
    const float x3 = fmul(fmul(fmul(0.044715f, x), x), x);
    const float t = tanhf_glibc(fmul(k, fadd(x, x3)));
    return fmul(fmul(0.5f, x), fadd(1.0f, t));
  }
};
// ops.rs:286-289: grad_b = g * ((-a) / (b*b))
RT_HD float div_grad_b(float g, float a, float b) { return fmul(g, fdiv(-a, fmul(b, b))); }

struct GradDivB {
  RT_HD float operator()(float g, float a, float b) const { return div_grad_b(g, a, b); }
};
// ops.rs:271-289: {g / b, g * ((-a) / (b*b))}
struct GradDiv2 {
  RT_HD float2 operator()(float g, float a, float b) const {
    return make_float2(fdiv(g, b), div_grad_b(g, a, b));
  }
};
// ops.rs:222-231: {g * b, g * a}
struct GradMul2 {
  RT_HD float2 operator()(float g, float a, float b) const {
    return make_float2(fmul(g, b), fmul(g, a));
  }
};
// ops.rs:137-146 / :179-188 (Tensor::neg is a sign flip, tensor/mod.rs:199)
struct GradAdd2 {
  RT_HD float2 operator()(float g) const { return make_float2(g, g); }
};
struct GradSub2 {
  RT_HD float2 operator()(float g) const { return make_float2(g, -g); }
};
struct OpNeg {
  RT_HD float operator()(float g) const { return -g; }
};
struct OpCopy {
  RT_HD float operator()(float g) const { return g; }
};

// Tensor::full(shape, v) with v read on the device from the one-element
// grad_output: SumBackward uses (f32)(f64)g, MeanBackward (f32)((f64)g / n)
// (ops.rs:506-507, :547-548).
__global__ void __launch_bounds__(kThreads)
fill_from_kernel(const float* g, float* out, size_t n, double divisor, int divide) {
  const double gv = (double)__ldg(g);
  const float v = divide ? (float)__ddiv_rn(gv, divisor) : (float)gv;
  const size_t n4 = n >> 2;
  float4* o4 = reinterpret_cast<float4*>(out);
  const bool vec = (reinterpret_cast<uintptr_t>(out) & 15u) == 0;
  const size_t start = vec ? n4 << 2 : 0;
  if (vec) {
    const float4 vv = make_float4(v, v, v, v);
    for (size_t j = (size_t)blockIdx.x * kThreads + threadIdx.x; j < n4;
         j += (size_t)gridDim.x * kThreads)
      __stcs(o4 + j, vv);
  }
  for (size_t i = start + (size_t)blockIdx.x * kThreads + threadIdx.x; i < n;
       i += (size_t)gridDim.x * kThreads)
    out[i] = v;
}

}  // namespace

cudaError_t launch_grad_unary(GradUnaryOp op, const float* g, const float* saved, float* out,
                              size_t n, cudaStream_t s) {
  In<2> in{{g, saved}};
  switch (op) {
    case kGradRelu: return launch_map(GradRelu{}, in, out, n, s);
    case kGradSigmoid: return launch_map(GradSigmoid{}, in, out, n, s);
    case kGradTanh: return launch_map(GradTanh{}, in, out, n, s);
    case kGradGelu: {
      volatile float three = 3.0f, c = 0.044715f;
      return launch_map(GradGelu{gelu_k(), three * c}, in, out, n, s);
    }
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_gelu_autograd(const float* x, float* out, size_t n, cudaStream_t s) {
  In<1> in{{x}};
  return launch_map(OpGeluAutograd{gelu_k()}, in, out, n, s);
}

cudaError_t launch_grad_binary(GradBinaryOp op, const float* g, const float* a, const float* b,
                               float* grad_a, float* grad_b, size_t n, cudaStream_t s) {
  if (n == 0 || (!grad_a && !grad_b)) return cudaSuccess;
  switch (op) {
    case kGradAdd:
    case kGradSub: {
      In<1> in{{g}};
      if (grad_a && grad_b)
        return op == kGradAdd ? launch_map2(GradAdd2{}, in, grad_a, grad_b, n, s)
                              : launch_map2(GradSub2{}, in, grad_a, grad_b, n, s);
      if (grad_a) return launch_map(OpCopy{}, in, grad_a, n, s);
      return op == kGradAdd ? launch_map(OpCopy{}, in, grad_b, n, s)
                            : launch_map(OpNeg{}, in, grad_b, n, s);
    }
    case kGradMul: {
      if (grad_a && grad_b) return launch_map2(GradMul2{}, In<3>{{g, a, b}}, grad_a, grad_b, n, s);
      if (grad_a) return launch_map(OpMul{}, In<2>{{g, b}}, grad_a, n, s);
      return launch_map(OpMul{}, In<2>{{g, a}}, grad_b, n, s);
    }
    case kGradDiv: {
      if (grad_a && grad_b) return launch_map2(GradDiv2{}, In<3>{{g, a, b}}, grad_a, grad_b, n, s);
      if (grad_a) return launch_map(OpDiv{}, In<2>{{g, b}}, grad_a, n, s);
      return launch_map(GradDivB{}, In<3>{{g, a, b}}, grad_b, n, s);
    }
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_fill_from(const float* g, float* out, size_t n, double divisor, bool divide,
                             cudaStream_t s) {
  if (n == 0) return cudaSuccess;
  fill_from_kernel<<<grid_for(std::max<size_t>(n >> 2, 1), kThreads), kThreads, 0, s>>>(
      g, out, n, divisor, divide ? 1 : 0);
  return cudaGetLastError();
}

}  // namespace rt
