"""The peer-memory all-reduce of the sharded sum's partials
(rtc_peer_allreduce_sum_f64, sharded.PeerSum).

On one GPU: a single rank returns its own value, and a wait for a rank that
never writes (a slot nothing sets) ends after the 2 s limit with NaN and the
error rtc_synchronize reports, leaving the context usable.  On two or more
GPUs: one process per GPU (spawned, gloo for the handle exchange) sums
distinct partials over several generations; every rank gets the rank-order
sum, bit for bit.
"""
import ctypes
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _lib():
    from rusttorch_b200 import _native as N
    return N, N.lib()


def _dev_alloc(N, lib, nbytes):
    p = ctypes.c_void_p()
    N.check(lib.rtc_malloc(0, nbytes, ctypes.byref(p)))
    zero = (ctypes.c_char * nbytes)()
    N.check(lib.rtc_memcpy_h2d(0, p, zero, nbytes))
    return p


def _put_f64(N, lib, p, v):
    b = np.array([v], dtype=np.float64)
    N.check(lib.rtc_memcpy_h2d(0, p, b.ctypes.data, 8))


def _get_f64(N, lib, p):
    b = np.zeros(1, dtype=np.float64)
    N.check(lib.rtc_memcpy_d2h(0, b.ctypes.data, p, 8))
    return float(b[0])


def test_single_rank_returns_its_value():
    N, lib = _lib()
    N.check(lib.rtc_set_device(0))
    slots = _dev_alloc(N, lib, lib.rtc_peer_slot_bytes(1))
    local, out = _dev_alloc(N, lib, 8), _dev_alloc(N, lib, 8)
    ptrs = (ctypes.c_void_p * 1)(slots.value)
    try:
        for g, v in ((1, 3.25), (2, -1e300), (3, 0.1)):
            _put_f64(N, lib, local, v)
            N.check(lib.rtc_peer_allreduce_sum_f64(0, local, ptrs, 1, 0, g, out))
            N.check(lib.rtc_synchronize())
            assert _get_f64(N, lib, out) == 0.0 + v
    finally:
        for p in (slots, local, out):
            N.check(lib.rtc_free(0, p))


def test_missing_rank_times_out_with_an_error():
    """Rank 0 of two, where rank 1's value never arrives (its slot in rank
    0's array is never written): the kernel gives up after 2 s."""
    import time
    N, lib = _lib()
    N.check(lib.rtc_set_device(0))
    nbytes = lib.rtc_peer_slot_bytes(2)
    mine, other = _dev_alloc(N, lib, nbytes), _dev_alloc(N, lib, nbytes)
    local, out = _dev_alloc(N, lib, 8), _dev_alloc(N, lib, 8)
    ptrs = (ctypes.c_void_p * 2)(mine.value, other.value)
    try:
        _put_f64(N, lib, local, 1.0)
        t0 = time.time()
        N.check(lib.rtc_peer_allreduce_sum_f64(0, local, ptrs, 2, 0, 1, out))
        with pytest.raises(N.RusttorchError) as e:
            N.check(lib.rtc_synchronize())
        assert e.value.code == N.BACKEND_ERROR
        assert 1.5 < time.time() - t0 < 30
        assert np.isnan(_get_f64(N, lib, out))
        N.check(lib.rtc_synchronize())   # the flag was taken; the context still works
    finally:
        for p in (mine, other, local, out):
            N.check(lib.rtc_free(0, p))


def _rank_main(rank, world, port, q):
    try:
        import torch
        import torch.distributed as dist

        torch.cuda.set_device(rank)
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        from rusttorch_b200 import _native as N
        from rusttorch_b200 import sharded as sh
        lib = N.lib()
        N.check(lib.rtc_set_device(rank))
        peer = sh.PeerSum(lib, rank, world, rank)
        local = torch.zeros(1, dtype=torch.float64, device="cuda")
        out = torch.zeros(1, dtype=torch.float64, device="cuda")
        got = []
        for g in range(5):
            vals = [0.1 * (r + 1) + 1e-17 * g + 2.0 ** (-40 + r) for r in range(world)]
            local.fill_(vals[rank])
            torch.cuda.synchronize()
            peer.allreduce(local.data_ptr(), out.data_ptr())
            N.check(lib.rtc_synchronize())
            want = 0.0
            for v in vals:
                want = want + v
            got.append((float(out.item()), want))
        peer.close()
        dist.destroy_process_group()
        q.put((rank, got, None))
    except Exception as ex:  # reported to the parent
        q.put((rank, None, repr(ex)))


@pytest.mark.parametrize("world", [2, 4, 8])
def test_ranks_on_separate_gpus_get_the_rank_order_sum(world):
    import multiprocessing as mp
    import torch
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    for _ in range(world):
        rank, got, err = q.get(timeout=180)
        results[rank] = (got, err)
    for p in procs:
        p.join(timeout=60)
    for rank, (got, err) in results.items():
        assert err is None, (rank, err)
        for value, want in got:
            assert value == want, (rank, value, want)
