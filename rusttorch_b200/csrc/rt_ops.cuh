// rt_ops.cuh — per-element rules of rusttorch-core's hot path, one functor per
// reference op, each keeping the reference's f32 operation order with one
// rounding per operation (rt::fadd/fmul/... are the _rn intrinsics on the
// device).  Citations are to rusttorch-core/src/ops/.
#pragma once

#include "rt_libm.cuh"

namespace rt {

// ---- binary: elementwise.rs:14 add, :97 mul, :130 sub, :163 div ----------
struct OpAdd { RT_HD float operator()(float a, float b) const { return fadd(a, b); } };
struct OpSub { RT_HD float operator()(float a, float b) const { return fsub(a, b); } };
struct OpMul { RT_HD float operator()(float a, float b) const { return fmul(a, b); } };
struct OpDiv { RT_HD float operator()(float a, float b) const { return fdiv(a, b); } };
// add followed by mul_scalar (elementwise.rs:14 then :213), fused in one pass.
struct OpAddMulScalar {
  float s;
  RT_HD float operator()(float a, float b) const { return fmul(fadd(a, b), s); }
};

// ---- scalar: elementwise.rs:200 add_scalar, :213 mul_scalar --------------
struct OpAddScalar {
  static constexpr bool kLight = true;
  float s;
  RT_HD float operator()(float x) const { return fadd(x, s); }
};
struct OpMulScalar {
  static constexpr bool kLight = true;
  float s;
  RT_HD float operator()(float x) const { return fmul(x, s); }
};

// ---- ternary: simd.rs:275 fused_multiply_add = a*b + c, two roundings ------
struct OpFma {
  RT_HD float operator()(float a, float b, float c) const { return fadd(fmul(a, b), c); }
};

// ---- activations: activation.rs -------------------------------------------
// :8 relu = x.max(0.0): maxnum(x, 0.0) lowers to (x > 0 ? x : 0.0) on x86_64,
// so NaN -> +0 and -0 -> +0.
struct OpRelu {
  static constexpr bool kLight = true;
  RT_HD float operator()(float x) const { return x > 0.0f ? x : 0.0f; }
};
// :170 leaky_relu
struct OpLeakyRelu {
  static constexpr bool kLight = true;
  float alpha;
  RT_HD float operator()(float x) const { return x > 0.0f ? x : fmul(alpha, x); }
};
// :21 sigmoid = 1 / (1 + exp(-x))
struct OpSigmoid {
  RT_HD float operator()(float x) const { return frcp(fadd(1.0f, expf_glibc(-x))); }
};
// :40 tanh
struct OpTanh {
  static constexpr bool kHeavy = true;
  RT_HD float operator()(float x) const { return tanhf_glibc(x); }
};
// :61 gelu = (0.5*x) * (1 + tanh(k*(x + 0.044715*((x*x)*x)))), k = sqrt(2/pi) in f32
struct OpGelu {
  static constexpr bool kHeavy = true;
  float k;
  RT_HD float operator()(float x) const {
    const float x3 = fmul(fmul(x, x), x);
    const float inner = fadd(x, fmul(0.044715f, x3));
    const float t = tanhf_glibc(fmul(k, inner));
    return fmul(fmul(0.5f, x), fadd(1.0f, t));
  }
};
// :263 swish (SiLU) = x / (1 + exp(-x))
struct OpSwish {
  RT_HD float operator()(float x) const { return fdiv(x, fadd(1.0f, expf_glibc(-x))); }
};
// :195 elu = x > 0 ? x : alpha*(exp(x) - 1)
struct OpElu {
  float alpha;
  RT_HD float operator()(float x) const {
    return x > 0.0f ? x : fmul(alpha, fsub(expf_glibc(x), 1.0f));
  }
};
// :228 selu = SCALE * (x > 0 ? x : ALPHA*(exp(x) - 1)), f64 constants cast to f32
struct OpSelu {
  float alpha, scale;
  RT_HD float operator()(float x) const {
    const float inner = x > 0.0f ? x : fmul(alpha, fsub(expf_glibc(x), 1.0f));
    return fmul(scale, inner);
  }
};
// :319 softplus = x > 20 ? x : ln(1 + exp(x))
RT_HD float softplus1(float x) {
  // 1 + exp(x) is in [1, 4.9e8] or NaN when x <= 20, so logf_pos applies
  return x > 20.0f ? x : logf_pos(fadd(1.0f, expf_glibc(x)));
}
struct OpSoftplus {
  static constexpr bool kHeavy = true;
  RT_HD float operator()(float x) const { return softplus1(x); }
};
// :284 mish = x * tanh(softplus(x))
struct OpMish {
  static constexpr bool kHeavy = true;
  RT_HD float operator()(float x) const { return fmul(x, tanhf_glibc(softplus1(x))); }
};
// :351 softsign = x / (1 + |x|)
struct OpSoftsign {
  RT_HD float operator()(float x) const { return fdiv(x, fadd(1.0f, fabsf(x))); }
};

// ---- ordering rules of Iterator::max_by / min_by with partial_cmp ---------
// (reduction.rs:36-40, :58-62; activation.rs:111-116).  Unordered compares
// Equal; Equal keeps the later element for max and the earlier for min.
RT_HD float max_fold(float acc, float x) { return acc > x ? acc : x; }
RT_HD float min_fold(float acc, float x) { return acc > x ? x : acc; }

}  // namespace rt
