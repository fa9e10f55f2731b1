"""Derives the polynomial coefficients of rt_fastmath.cuh (run by hand; the
header holds the printed values).

Each polynomial is a Chebyshev-series fit (mpmath.chebyfit, 50 digits) of
the smooth remainder of a function after its exactly known leading terms,
on the interval the header's argument reduction leaves, with every
coefficient then rounded to float32:

  exp:  e^r = 1 + r + r^2 * E(r),        E(r) = (e^r - 1 - r) / r^2,
        r in [-ln2/2, ln2/2] (+ margin for the reduction's rounding);
  tanh: tanh(x) = x + x^3 * T(x^2),       T(u) = (tanh(sqrt u) - sqrt u) / u^1.5,
        |x| < 0.55;
  log:  log(1 + f) = f + f^2 * (-1/2 + f * L(f)),
        L(f) = (log1p(f) - f + f^2/2) / f^3, f = m - 1, m in [sqrt(2)/2, sqrt(2)).

It prints each polynomial's coefficients (highest degree first, as the
header's Horner steps use them) and the largest relative error of the
float32-rounded polynomial over 20001 points of its interval, evaluated in
50-digit arithmetic (the rounding of the float32 evaluation itself is
checked exhaustively by tests/native/fastmath_check.cpp).
"""
from __future__ import annotations

import struct

import mpmath as mp

mp.mp.dps = 50


def f32(v) -> float:
    return struct.unpack("<f", struct.pack("<f", float(v)))[0]


def hexf(v: float) -> str:
    return "0x%08x" % struct.unpack("<I", struct.pack("<f", v))[0]


def fit(fn, a, b, n):
    coeffs, err = mp.chebyfit(fn, [a, b], n, error=True)
    return [f32(c) for c in coeffs], err       # highest degree first


def horner(cs, x):
    acc = mp.mpf(0)
    for c in cs:
        acc = acc * x + mp.mpf(c)
    return acc


def report(name, cs, true_fn, approx_fn, a, b):
    worst = mp.mpf(0)
    for i in range(20001):
        x = mp.mpf(a) + (mp.mpf(b) - mp.mpf(a)) * i / 20000
        if x == 0:
            continue
        t = true_fn(x)
        worst = max(worst, abs((approx_fn(x) - t) / t))
    print(f"{name}: max relative error of the f32 polynomial {mp.nstr(worst, 4)} "
          f"({mp.nstr(worst / mp.mpf(2) ** -24, 3)} half-ulps)")
    for c in cs:
        print(f"  {c!r:>24}  {hexf(c)}")


def main() -> None:
    half_ln2 = mp.log(2) / 2 + mp.mpf("1e-6")
    e_cs, _ = fit(lambda r: (mp.exp(r) - 1 - r) / r**2 if r != 0 else mp.mpf(0.5),
                  -half_ln2, half_ln2, 5)
    report("exp E(r), degree 4", e_cs, mp.exp,
           lambda r: 1 + r + r * r * horner(e_cs, r), -half_ln2, half_ln2)

    xt = mp.mpf("0.55")
    t_cs, _ = fit(lambda u: (mp.tanh(mp.sqrt(u)) - mp.sqrt(u)) / u**1.5 if u != 0
                  else mp.mpf(-1) / 3, mp.mpf(0), xt * xt, 5)
    report("tanh T(u), degree 4", t_cs, mp.tanh,
           lambda x: x + x**3 * horner(t_cs, x * x), mp.mpf("1e-4"), xt)

    lo, hi = mp.sqrt(2) / 2 - 1, mp.sqrt(2) - 1
    l_cs, _ = fit(lambda f: (mp.log1p(f) - f + f * f / 2) / f**3 if f != 0 else mp.mpf(1) / 3,
                  lo, hi, 8)
    report("log L(f), degree 7", l_cs, mp.log1p,
           lambda f: f + f * f * (mp.mpf(-0.5) + f * horner(l_cs, f)), lo, hi)


if __name__ == "__main__":
    main()
