// rt_fastmath.cuh — float32 exp, tanh, log and reciprocal for the
// tolerance math mode of the activations.
//
// north_star holds the transcendental activations and softmax to the
// reference's results within 1e-6 relative error or 4 ulp, not bit for bit.
// The bit-exact restatement of glibc (rt_libm.cuh) spends most of its
// instructions in double-precision table steps; these functions reach the
// tolerance in single precision, so the kernels that use them stay bound by
// HBM rather than by instruction issue.
//
// Methods (all single precision, one rounding per operation, so the host
// build below is bit-identical to the device build and the host can check
// every one of the 2^32 inputs against glibc):
//  * exp — Cody and Waite's argument reduction x = k*ln2 + r (k by the
//    round-to-nearest shift 1.5*2^23, ln2 split into a float and the float
//    of the remainder, r from two fused multiply-adds), e^r on
//    [-ln2/2, ln2/2] as 1 + r + r^2*E(r) with E a degree-4 Chebyshev fit
//    (gen_fastmath.py), and 2^k applied as two exact power-of-two factors so
//    that results in the subnormal range are rounded once;
//  * tanh — an odd polynomial x + x^3*T(x^2) below |x| = 0.55, and
//    1 - 2/(e^(2|x|) + 1) above;
//  * log — x = 2^k * m with m in [sqrt(1/2), sqrt(2)), f = m - 1 (exact),
//    log(1 + f) = f + f^2*(-1/2 + f*L(f)) with L a degree-7 Chebyshev fit,
//    plus k*ln2 in two parts;
//  * reciprocal — the hardware approximation refined by two Newton-Raphson
//    steps y' = y + y*(1 - d*y) (fused), which is the correctly rounded 1/d
//    for every d in [1, 2^64] (rcp_rn in rt_libm.cuh; tests/test_tolerance_gpu.py
//    checks it against IEEE division on the device); the host build divides.
#pragma once

#include "rt_libm.cuh"

namespace rt {

RT_HD float ffma(float a, float b, float c) {
#if defined(__CUDA_ARCH__)
  return __fmaf_rn(a, b, c);
#else
  return fmaf(a, b, c);
#endif
}

RT_HD float fabs_bits(float x) { return u2f(f2u(x) & 0x7fffffffu); }

// 1/d rounded to nearest for d in [1, 2^64] (and NaN for NaN): rcp_rn.
RT_HD float rcp_cr(float d) { return rcp_rn(d); }

// e^x = p * s1 * s2 for x in [-104, 89] (or NaN): p in [0.70, 1.42] and s1,
// s2 powers of two (each in [2^-75, 2^64]).  Callers that scale the result
// multiply p by their factors first and apply s1, s2 last, so a result in
// the subnormal range is rounded once.
struct ExpParts {
  float p, s1, s2;
};

// e^x = p * 2^k (p in [0.70, 1.42]) for x in [-104, 89] (or NaN).
RT_HD float exp_core(float x, int* kout) {
  const float kLog2e = u2f(0x3fb8aa3bu);
  const float kShift = 12582912.0f;           // 1.5 * 2^23
  const float kLn2Hi = u2f(0x3f317218u);      // ln2 rounded to float
  const float kLn2Lo = u2f(0xb102e308u);      // ln2 - kLn2Hi rounded to float
  // E(r) = (e^r - 1 - r)/r^2, highest degree first (gen_fastmath.py)
  const float kE4 = u2f(0x3ab6887eu), kE3 = u2f(0x3c0905b1u), kE2 = u2f(0x3d2aaa8du);
  const float kE1 = u2f(0x3e2aaa6fu), kE0 = 0.5f;
  const float t = ffma(x, kLog2e, kShift);    // 1.5*2^23 + round(x*log2(e))
  const float kf = fsub(t, kShift);
  const int k = (int)(f2u(t) - 0x4b400000u);
  float r = ffma(kf, -kLn2Hi, x);             // exact
  r = ffma(kf, -kLn2Lo, r);
  float h = ffma(kE4, r, kE3);
  h = ffma(h, r, kE2);
  h = ffma(h, r, kE1);
  h = ffma(h, r, kE0);
  h = ffma(h, r, 1.0f);                       // 1 + r*E(r)
  *kout = k;
  return ffma(h, r, 1.0f);                    // 1 + r + r^2*E(r)
}

RT_HD ExpParts exp_parts(float x) {
  int k;
  const float p = exp_core(x, &k);
  const int k1 = k >> 1, k2 = k - k1;
  return ExpParts{p, u2f((uint32_t)(k1 + 127) << 23), u2f((uint32_t)(k2 + 127) << 23)};
}

// e^x for any float x: +inf above 89, +0 below -104 (both clamps keep NaN).
RT_HD float exp_fast(float x) {
  const float lo = x < -104.0f ? -104.0f : x;
  const ExpParts e = exp_parts(lo > 89.0f ? 89.0f : lo);
  return fmul(fmul(e.p, e.s1), e.s2);
}

// e^x for x <= 0 or NaN (softmax's x - max): +0 below -104.
RT_HD float exp_fast_nonpos(float x) {
  const ExpParts e = exp_parts(x < -104.0f ? -104.0f : x);
  return fmul(fmul(e.p, e.s1), e.s2);
}

// tanh(x) for any float x (odd; +-1 beyond |x| = 9.02, where the rounded
// result is +-1).
RT_HD float tanh_fast(float x) {
  // T(u) = (tanh(sqrt u) - sqrt u)/u^1.5, highest degree first
  const float kT4 = u2f(0xbbd89a9cu), kT3 = u2f(0x3cae9107u), kT2 = u2f(0xbd5cd022u);
  const float kT1 = u2f(0x3e0887f5u), kT0 = u2f(0xbeaaaaaau);
  const uint32_t sign = f2u(x) & 0x80000000u;
  const float ax = fabs_bits(x);
  const float x2 = fmul(ax, ax);
  float h = ffma(kT4, x2, kT3);
  h = ffma(h, x2, kT2);
  h = ffma(h, x2, kT1);
  h = ffma(h, x2, kT0);
  const float small = ffma(fmul(ax, x2), h, ax);
  // 1 - 2/(e^(2|x|) + 1); e^19 + 1 < 2^64 keeps rcp_cr in range
  const ExpParts e = exp_parts(fmul(2.0f, ax > 9.5f ? 9.5f : ax));
  const float big = ffma(-2.0f, rcp_cr(fadd(fmul(fmul(e.p, e.s1), e.s2), 1.0f)), 1.0f);
  const float r = ax < 0.55f ? small : big;
  return u2f(f2u(r) | sign);
}

// tanh(z) to within a few units of 2^-24 in ABSOLUTE terms, which is all
// GELU needs of it above its exact range (it only uses 1 + tanh(z), which is
// above 0.1 there): tanh_fast's large-|z| formula 1 - 2/(e^(2|z|) + 1) on
// every input, so no small-|z| polynomial; near 0 its cancellation costs
// relative accuracy of tanh itself, not absolute.
RT_HD float tanh_fast_abs(float z) {
  const float az = fabs_bits(z);
  // 2|z| <= 19, so 2^k with k <= 28 is one normal power of two: e = p * 2^k.
  int k;
  const float p = exp_core(fmul(2.0f, az > 9.5f ? 9.5f : az), &k);
  const float t = ffma(-2.0f, rcp_cr(fadd(fmul(p, u2f((uint32_t)(k + 127) << 23)), 1.0f)), 1.0f);
  return u2f(f2u(t) | (f2u(z) & 0x80000000u));
}

// log(y) for a positive normal finite y (garbage, but no fault, for other
// inputs, NaN included: callers that can see a NaN use log_fast).
RT_HD float log_fast_pos(float y) {
  const float kLn2Hi = u2f(0x3f317218u), kLn2Lo = u2f(0xb102e308u);
  // L(f) = (log1p(f) - f + f^2/2)/f^3, highest degree first
  const float kL7 = u2f(0xbda1d923u), kL6 = u2f(0x3e0140a7u), kL5 = u2f(0xbe0519f5u);
  const float kL4 = u2f(0x3e118e73u), kL3 = u2f(0xbe2a681fu), kL2 = u2f(0x3e4ccf8au);
  const float kL1 = u2f(0xbe800067u), kL0 = u2f(0x3eaaaaaau);
  const uint32_t iy = f2u(y);
  const uint32_t tmp = iy - 0x3f3504f3u;              // sqrt(1/2) rounded to float
  const int k = (int32_t)tmp >> 23;
  const float f = fsub(u2f(iy - (tmp & 0xff800000u)), 1.0f);   // m - 1, exact
  float h = ffma(kL7, f, kL6);
  h = ffma(h, f, kL5);
  h = ffma(h, f, kL4);
  h = ffma(h, f, kL3);
  h = ffma(h, f, kL2);
  h = ffma(h, f, kL1);
  h = ffma(h, f, kL0);
  const float l = ffma(fmul(f, f), ffma(h, f, -0.5f), f);
  const float kf = (float)k;
  return ffma(kf, kLn2Hi, ffma(kf, kLn2Lo, l));
}

// log(y) for a positive normal finite y, or NaN for NaN.
RT_HD float log_fast(float y) {
  const float r = log_fast_pos(y);
  return y != y ? y : r;
}

}  // namespace rt
