// rt_ops.cuh — per-element rules of rusttorch-core's hot path, one functor per
// reference op, each keeping the reference's f32 operation order with one
// rounding per operation (rt::fadd/fmul/... are the _rn intrinsics on the
// device).  Citations are to rusttorch-core/src/ops/.
#pragma once

#include "rt_fastmath.cuh"
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

// ---- the same activations in the tolerance math mode ---------------------
// Within north_star's 1e-6 relative error or 4 ulp of the reference's formula
// over glibc, on every float input (tests/native/fastmath_check.cpp), from
// the single-precision functions of rt_fastmath.cuh.
//
// glibc's expf(t) is +inf exactly for t >= 88.72283935546875 (0x42b17218),
// so the reference's 1/(1 + exp(-x)) is +0 and x/(1 + exp(-x)) is -0 for
// x <= -88.72283935546875; below that the result would otherwise be a tiny
// nonzero value.
constexpr float kExpOverflowNeg = -88.72283935546875f;

// :21 sigmoid.  With e = exp(-|x|): 1/(1 + e) for x >= 0 and e/(1 + e) for
// x < 0 (the same value; the second form never overflows, and its result,
// scaled last, is rounded once when it is subnormal).
struct OpSigmoidTol {
  RT_HD float operator()(float x) const {
    const float na = u2f(f2u(x) | 0x80000000u);          // -|x|
    const ExpParts e = exp_parts(na < -104.0f ? -104.0f : na);
    const float r = rcp_cr(fadd(1.0f, fmul(fmul(e.p, e.s1), e.s2)));
    const float y = x < 0.0f ? fmul(fmul(fmul(e.p, r), e.s1), e.s2) : r;
    return x <= kExpOverflowNeg ? 0.0f : y;
  }
};
// :263 swish = x/(1 + exp(-x)), the same way (x*e/(1 + e) for x < 0).
struct OpSwishTol {
  RT_HD float operator()(float x) const {
    const float na = u2f(f2u(x) | 0x80000000u);
    const ExpParts e = exp_parts(na < -104.0f ? -104.0f : na);
    const float r = rcp_cr(fadd(1.0f, fmul(fmul(e.p, e.s1), e.s2)));
    const float y = x < 0.0f ? fmul(fmul(fmul(fmul(e.p, r), x), e.s1), e.s2) : fmul(x, r);
    return x <= kExpOverflowNeg ? fmul(x, 0.0f) : y;
  }
};
// :40 tanh
struct OpTanhTol {
  RT_HD float operator()(float x) const { return tanh_fast(x); }
};
// :319 softplus = x > 20 ? x : ln(1 + exp(x)).  1 + exp(x) is the
// reference's float bit for bit (expf_glibc): for x well below 0 its last bit
// decides the result's leading digits, and only the log is approximated.
struct OpSoftplusTol {
  static constexpr bool kHeavy = true;   // one vector per thread per iteration
  RT_HD float operator()(float x) const {
    // !(x <= 20): x > 20, or x NaN (returned as is); below, 1 + exp(x) is a
    // positive normal float in [1, 4.9e8]
    return !(x <= 20.0f) ? x : log_fast_pos(fadd(1.0f, expf_glibc_le89(x)));
  }
};
// :284 mish = x * tanh(softplus(x)).  With y = 1 + exp(x) (the reference's
// float, as in softplus), tanh(ln y) = (y^2 - 1)/(y^2 + 1) =
// (y - 1)(y + 1)/(y*y + 1): no log and no tanh, and y - 1 is exact.  For
// x > 20 the reference's tanh(x) is 1, so mish is x.
struct OpMishTol {
  RT_HD float operator()(float x) const {
    const float y = fadd(1.0f, expf_glibc_le89(x));   // exp(x) is used only for x <= 20
    const float num = fmul(fsub(y, 1.0f), fadd(y, 1.0f));
    const float t = fmul(num, rcp_cr(ffma(y, y, 1.0f)));
    return x > 20.0f ? x : fmul(x, t);
  }
};

// :61 gelu.  1 + tanh(z) cancels for z well below 0: there the reference's
// result is the gap between -1 and glibc's tanhf(z), and it carries no more
// than a few of tanhf's bits, so tanhf must be glibc's to the last bit
// (tanhf_glibc).  Above kGeluExactBelow (1 + tanh(z) > 0.115) the
// cancellation magnifies the fast tanh's error by less than 9 and the result
// stays within 5.8e-7 of the reference's; below -9.1 glibc's tanhf is
// exactly -1.  The kernel sends only the middle range through
// tanhf_glibc (rt_map.cuh, map_split_kernel).
#ifndef RT_GELU_EXACT_BELOW
#define RT_GELU_EXACT_BELOW -1.4f
#endif
constexpr float kGeluExactBelow = RT_GELU_EXACT_BELOW;
struct OpGeluTol {
  float k;
  // z = k*(x + 0.044715*x^3), in the reference's order
  RT_HD float arg(float x) const {
    const float x3 = fmul(fmul(x, x), x);
    return fmul(k, fadd(x, fmul(0.044715f, x3)));
  }
  RT_HD static bool needs_exact(float z) { return z < kGeluExactBelow && z >= -9.1f; }
  // -1 exactly below -8.9 (2/(e^(2|z|) + 1) < 2^-25 there), as glibc's tanhf
  RT_HD static float fast_tanh(float z) { return tanh_fast_abs(z); }
  RT_HD static float exact_tanh(float z) { return tanhf_glibc_ge1(z); }   // 1.4 < |z| <= 9.1
  RT_HD static float finish(float x, float t) { return fmul(fmul(0.5f, x), fadd(1.0f, t)); }
  RT_HD float operator()(float x) const {
    const float z = arg(x);
    return finish(x, needs_exact(z) ? exact_tanh(z) : fast_tanh(z));
  }
};

// ---- ordering rules of Iterator::max_by / min_by with partial_cmp ---------
// (reduction.rs:36-40, :58-62; activation.rs:111-116).  Unordered compares
// Equal; Equal keeps the later element for max and the earlier for min.
RT_HD float max_fold(float acc, float x) { return acc > x ? acc : x; }
RT_HD float min_fold(float acc, float x) { return acc > x ? x : acc; }

}  // namespace rt
