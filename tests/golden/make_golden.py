"""Generate tests/golden/golden.npz: small input/expected-output fixtures.

The expected values come from an implementation independent of oracle/: plain
Python and numpy float32 scalars, restating each reference op (rusttorch-core
src/ops/*.rs) in its f32 order.  Transcendentals use Python's math module in
double precision rounded once to float32 (the reference calls glibc, which is
within 1 ulp of that), so the tests compare those ops within a few ulp and
everything else bit for bit.

The reference itself (Rust) cannot be built in this environment, and it ships
no golden vectors; these fixtures therefore pin the C oracle against a second,
separately written restatement.

    python tests/golden/make_golden.py
"""
from __future__ import annotations

import math
from pathlib import Path

import numpy as np

F = np.float32
OUT = Path(__file__).resolve().parent / "golden.npz"


def f(x) -> np.float32:
    return np.float32(x)


def r32(x: float) -> np.float32:
    """Round a Python float (double) once to float32."""
    return np.float32(x)


def edge_values() -> np.ndarray:
    vals = [0.0, -0.0, 1.0, -1.0, 0.5, -0.5, 2.0, -2.0, 1e-8, -1e-8, 3.5, -3.5, 10.0, -10.0,
            20.0, 20.5, -20.0, 1e-30, -1e-30, 0.1, -0.1, 7.25, -7.25, 15.0, -15.0]
    return np.array(vals, dtype=F)


def main() -> None:
    rng = np.random.default_rng(20261201)
    n = 257
    a = np.concatenate([edge_values(), (rng.standard_normal(n) * 3).astype(F)])
    b = np.concatenate([edge_values()[::-1], (rng.standard_normal(n) * 3).astype(F)])
    c = (rng.standard_normal(a.size)).astype(F)
    b_nz = np.where(b == 0, F(0.75), b).astype(F)
    g = {}
    g["a"], g["b"], g["c"], g["b_nz"] = a, b, c, b_nz

    # ---- elementwise, bit-exact (IEEE f32, one rounding per op) ----------
    g["add"] = (a + b).astype(F)
    g["sub"] = (a - b).astype(F)
    g["mul"] = (a * b).astype(F)
    g["div"] = (a / b_nz).astype(F)
    g["add_scalar"] = (a + F(10.0)).astype(F)
    g["mul_scalar"] = (a * F(0.5)).astype(F)
    g["add_mul_scalar"] = ((a + b).astype(F) * F(0.5)).astype(F)
    g["fma"] = ((a * b).astype(F) + c).astype(F)
    g["relu"] = np.array([x if x > 0 else F(0.0) for x in a], dtype=F)
    g["leaky_relu"] = np.array([x if x > 0 else F(0.01) * x for x in a], dtype=F)
    g["softsign"] = np.array([x / (F(1.0) + abs(x)) for x in a], dtype=F)

    # ---- transcendental (compared within a few ulp) ------------------------
    def sig(x):
        return F(1.0) / (F(1.0) + r32(math.exp(-float(x))))

    def swish(x):
        return x / (F(1.0) + r32(math.exp(-float(x))))

    k = r32(math.sqrt(float(F(2.0) / F(math.pi))))

    def gelu(x):
        x3 = (x * x) * x
        inner = x + F(0.044715) * x3
        t = r32(math.tanh(float(k * inner)))
        return (F(0.5) * x) * (F(1.0) + t)

    def elu(x, alpha=F(1.0)):
        return x if x > 0 else alpha * (r32(math.exp(float(x))) - F(1.0))

    def selu(x):
        return F(1.0507009873554805) * (x if x > 0 else F(1.6732632423543772) *
                                       (r32(math.exp(float(x))) - F(1.0)))

    def softplus(x):
        if x > F(20.0):
            return x
        return r32(math.log(float(F(1.0) + r32(math.exp(float(x))))))

    def mish(x):
        return x * r32(math.tanh(float(softplus(x))))

    with np.errstate(over="ignore"):
        g["sigmoid"] = np.array([sig(x) for x in a], dtype=F)
        g["swish"] = np.array([swish(x) for x in a], dtype=F)
        g["tanh"] = np.array([r32(math.tanh(float(x))) for x in a], dtype=F)
        g["gelu"] = np.array([gelu(x) for x in a], dtype=F)
        g["elu"] = np.array([elu(x) for x in a], dtype=F)
        g["selu"] = np.array([selu(x) for x in a], dtype=F)
        g["softplus"] = np.array([softplus(x) for x in a], dtype=F)
        g["mish"] = np.array([mish(x) for x in a], dtype=F)

    # ---- reductions ---------------------------------------------------------
    s = 0.0
    for x in a:
        s = s + float(x)          # sequential f64 fold (reduction.rs:9)
    g["sum"] = np.array([s])
    g["mean"] = np.array([s / a.size])

    def fold_max(xs):
        acc = xs[0]
        for x in xs[1:]:
            acc = acc if acc > x else x
        return acc

    def fold_min(xs):
        acc = xs[0]
        for x in xs[1:]:
            acc = x if acc > x else acc
        return acc

    g["max"] = np.array([fold_max(list(a))], dtype=F)
    g["min"] = np.array([fold_min(list(a))], dtype=F)

    def unrolled(xs):
        p = [F(0.0)] * 8
        i = 0
        while len(xs) - i >= 8:
            for j in range(8):
                p[j] = F(p[j] + xs[i + j])
            i += 8
        acc = F(0.0)
        acc = F(acc + F(p[0] + p[4]))
        acc = F(acc + F(p[1] + p[5]))
        acc = F(acc + F(p[2] + p[6]))
        acc = F(acc + F(p[3] + p[7]))
        for x in xs[i:]:
            acc = F(acc + x)
        return acc

    m2 = (rng.standard_normal((13, 37)) * 2).astype(F)
    g["m2"] = m2
    g["sum_dim1"] = np.array([unrolled(list(row)) for row in m2], dtype=F)
    col = np.zeros(m2.shape[1], dtype=F)
    for row in m2:
        col = (col + row).astype(F)   # res = res + row
    g["sum_dim0"] = col
    g["mean_dim1"] = np.array([unrolled(list(row)) / F(m2.shape[1]) for row in m2], dtype=F)
    g["mean_dim0"] = (col / F(m2.shape[0])).astype(F)
    g["max_dim1"] = np.array([fold_max(list(row)) for row in m2], dtype=F)
    g["max_dim0"] = np.array([fold_max(list(m2[:, j])) for j in range(m2.shape[1])], dtype=F)

    # softmax over the last dim
    sm = np.empty_like(m2)
    for i, row in enumerate(m2):
        mx = fold_max(list(row))
        e = [r32(math.exp(float(F(x - mx)))) for x in row]
        ssum = unrolled(e)
        sm[i] = [F(v / ssum) for v in e]
    g["softmax_dim1"] = sm

    # ---- AdamW (optimizer.rs:207-440), f32 order ---------------------------
    p = (rng.standard_normal(n) * 0.02).astype(F)
    gr = (rng.standard_normal(n) * 1e-2).astype(F)
    m = (rng.standard_normal(n) * 1e-3).astype(F)
    v = (rng.random(n) * 1e-4).astype(F)
    lr, b1, b2, eps, wd, t = 1e-3, 0.9, 0.999, 1e-8, 0.01, 10
    bc1, bc2 = 1.0 - b1 ** t, 1.0 - b2 ** t
    fb1, fb2 = F(b1), F(b2)
    po, mo, vo = [], [], []
    for pi, gi, mi, vi in zip(p, gr, m, v):
        nm = F(F(mi * fb1) + F(gi * F(F(1.0) - fb1)))
        nv = F(F(vi * fb2) + F(F(gi * gi) * F(F(1.0) - fb2)))
        mh = F(nm / F(bc1))
        vh = F(nv / F(bc2))
        den = F(F(np.sqrt(vh)) + F(eps))
        pa = F(pi - F(F(mh / den) * F(lr)))
        po.append(F(pa - F(pi * F(lr * wd))))
        mo.append(nm)
        vo.append(nv)
    g.update(adam_p=p, adam_g=gr, adam_m=m, adam_v=v, adamw_p_out=np.array(po, dtype=F),
             adamw_m_out=np.array(mo, dtype=F), adamw_v_out=np.array(vo, dtype=F))
    np.savez_compressed(OUT, **g)
    print(f"wrote {OUT} ({len(g)} arrays)")


if __name__ == "__main__":
    main()
