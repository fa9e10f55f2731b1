"""Every float32 bit pattern through the GPU activations (opt-in:
RT_EXHAUSTIVE=1; a few minutes on a 16-core host).

The ops that restate glibc's expf/tanhf bit for bit (relu, leaky_relu,
sigmoid, tanh, GELU, SiLU, ELU, SELU, softsign) are compared with the oracle
(the reference's formulas over this machine's glibc) on all 2^32 inputs.
softplus and mish, whose log is this repository's correctly rounded one, are
compared with the same per-element rule built for the host (rt_ops.cuh
under g++), which tests/test_libm_restatement.py bounds against glibc (1 and
6 ulp) on all 2^32 inputs.  The oracle and the host rule run on every host
core in slices; the GPU takes each 2^27-input chunk in one call.
"""
import concurrent.futures as cf
import os

import numpy as np
import pytest

from tests import _oracle as O

pytestmark = [pytest.mark.gpu, pytest.mark.usefixtures("exact_math"),
              pytest.mark.skipif(os.environ.get("RT_EXHAUSTIVE") != "1",
                                 reason="exhaustive sweep: set RT_EXHAUSTIVE=1")]

CHUNK = 1 << 27
ORACLE_OPS = [("relu", ()), ("leaky_relu", (0.01,)), ("sigmoid", ()), ("tanh", ()),
              ("gelu", ()), ("swish", ()), ("elu", (1.0,)), ("selu", ()), ("softsign", ())]


def _sweep(op, extra, reference):
    """Compare rt.<op> with reference(x_slice, out_slice) over all inputs;
    returns (mismatches, first mismatching bit pattern or None)."""
    import rusttorch_b200 as rt
    threads = os.cpu_count() or 1
    bounds = np.linspace(0, CHUNK, threads + 1).astype(np.int64)
    bad, first = 0, None
    with cf.ThreadPoolExecutor(threads) as pool:
        for c in range(0, 1 << 32, CHUNK):
            u = np.arange(c, c + CHUNK, dtype=np.uint64).astype(np.uint32)
            x = u.view(np.float32)
            want = np.empty_like(x)
            list(pool.map(lambda i: reference(x[bounds[i]:bounds[i + 1]],
                                              want[bounds[i]:bounds[i + 1]]), range(threads)))
            got = getattr(rt, op)(rt.Tensor.from_numpy(x), *extra).to_numpy()
            diff = (got.view(np.uint32) != want.view(np.uint32)) & ~(np.isnan(got) & np.isnan(want))
            n = int(np.count_nonzero(diff))
            if n and first is None:
                first = int(u[np.flatnonzero(diff)[0]])
            bad += n
    return bad, first


@pytest.mark.parametrize("op,extra", ORACLE_OPS)
def test_every_input_matches_the_oracle(op, extra):
    O.lib()

    def ref(xs, out):
        out[...] = O.unary(op, np.ascontiguousarray(xs), *extra)

    bad, first = _sweep(op, extra, ref)
    assert bad == 0, f"{op}: {bad} inputs differ, first 0x{first:08x}"


@pytest.mark.parametrize("op", ["softplus", "mish"])
def test_every_input_matches_the_host_rule(op):
    from tests.test_libm_restatement import load_check_lib
    chk = load_check_lib()
    which = ["softplus", "mish"].index(op)

    def ref(xs, out):
        xs = np.ascontiguousarray(xs)
        res = np.empty_like(xs)
        chk.act_restated(which, xs.ctypes.data, res.ctypes.data, xs.size)
        out[...] = res

    bad, first = _sweep(op, (), ref)
    assert bad == 0, f"{op}: {bad} inputs differ from the host rule, first 0x{first:08x}"
