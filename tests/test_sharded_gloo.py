"""Sharded global reductions: the host-side logic on CPU ranks (gloo).

Two processes hold contiguous shards of one tensor, summarise them (here
with a Python restatement of the per-shard summary; the GPU test checks the
device summary against the same function), all-gather the 32-byte summaries
over gloo and fold them with the library's rtc_shard_combine.  The result
must equal the oracle's sum/mean/max/min of the whole tensor, including the
order-dependent max/min folds across shard boundaries.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from rusttorch_b200 import sharded
from tests import _oracle as O


def summary_of(x: np.ndarray) -> sharded.ShardSummary:
    """What rtc_shard_summary_local computes, restated with the oracle."""
    s = sharded.ShardSummary()
    s.count = x.size
    s.sum = O.sum(x) if x.size else 0.0
    s.min_nonnan = float("inf")
    if x.size == 0:
        return s
    nan = np.isnan(x)
    if nan.any():
        last = int(np.flatnonzero(nan)[-1])
        s.max_kind = 2
        s.max = float("nan") if last == x.size - 1 else O.scalar_reduce("max", x[last + 1:])[1]
    else:
        s.max_kind = 1
        s.max = O.scalar_reduce("max", x)[1]
    keep = x[~nan]
    if keep.size:
        s.min_nonnan = O.scalar_reduce("min", np.ascontiguousarray(keep))[1]
    s.first_nan = int(bool(nan[0]))
    return s


CASES = {
    "random": lambda: O.normal(10001, 9),
    "nan_in_first_shard": lambda: _plant(O.normal(1000, 9), {10: np.nan}),
    "nan_at_shard_end": lambda: _plant(O.normal(1000, 9), {499: np.nan}),
    "nan_first_element": lambda: _plant(O.normal(1000, 9), {0: np.nan}),
    "nan_starts_second": lambda: _plant(O.normal(1000, 9), {500: np.nan}),
    "zero_ties_across": lambda: np.array([-1, 0.0, -2, -0.0] * 2, dtype=np.float32),
    "zero_ties_across_rev": lambda: np.array([-0.0, -1, 0.0, -3] * 2, dtype=np.float32),
    "empty_second_shard": lambda: O.normal(7, 3),
}


def _plant(x, d):
    for k, v in d.items():
        x[k] = v
    return x


def _split(x, world, case):
    if case == "empty_second_shard":
        return [x, x[:0]]
    return np.array_split(x, world)


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    out = {}
    for name, make in CASES.items():
        x = make()
        mine = _split(x, world, name)[rank]
        s = summary_of(np.ascontiguousarray(mine))
        raw = torch.frombuffer(bytearray(bytes(s)), dtype=torch.uint8)
        gathered = [torch.empty_like(raw) for _ in range(world)]
        dist.all_gather(gathered, raw)
        parts = [sharded.ShardSummary.from_buffer_copy(t.numpy().tobytes()) for t in gathered]
        out[name] = sharded.combine(parts)
    dist.destroy_process_group()
    q.put((rank, out))


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_gloo_ranks_match_the_whole_tensor():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for name, make in CASES.items():
        x = make()
        want_sum = O.sum(x)
        want = {op: O.scalar_reduce(op, x)[1] for op in ("max", "min", "mean")}
        for rank in range(world):
            s, mean, mx, mn = results[rank][name]
            assert (np.isnan(s) and np.isnan(want_sum)) or \
                abs(s - want_sum) <= 1e-9 * max(1.0, float(np.nansum(np.abs(x)))), (name, s)
            for got, exp, op in ((mx, want["max"], "max"), (mn, want["min"], "min")):
                gb = np.float32(got).view(np.uint32)
                eb = np.float32(exp).view(np.uint32)
                assert (np.isnan(got) and np.isnan(exp)) or gb == eb, (name, op, got, exp)
        assert results[0][name] == pytest.approx(results[1][name], nan_ok=True)


def test_combine_of_empty_is_an_error():
    with pytest.raises(ValueError, match="empty tensor"):
        sharded.combine([sharded.ShardSummary()])


# ------------------------------------------------- a rank that leaves
# Failure detection on the host (no GPU is involved): two gloo ranks run the
# sharded reduction's exchange for one step; then rank 1 either stays alive
# without joining the next step or exits.  Rank 0's ShardedReducer, built
# with a short timeout, must raise instead of waiting for the process
# group's own timeout (set long here, 120 s, so it cannot be what ends it).
LIMIT_S = 3.0


def _leaving_worker(rank, world, port, mode, q):
    import time
    from datetime import timedelta

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    red = sharded.ShardedReducer(sharded.N.lib(), rank, world, timeout_s=LIMIT_S)
    s = summary_of(O.normal(1000, 7 + rank))
    first = red.exchange(s)                       # step 1: everyone takes part
    if rank == 1:
        if mode == "stays":
            time.sleep(LIMIT_S + 4)               # alive, never joins step 2
        os._exit(0)                               # or simply gone
    t0 = time.perf_counter()
    try:
        red.exchange(s)
        q.put(("no error", time.perf_counter() - t0, len(first)))
    except ValueError as e:
        q.put((getattr(e, "kind", type(e).__name__), time.perf_counter() - t0, str(e)[:200]))
    q.close()
    q.join_thread()                               # deliver the result before leaving
    os._exit(0)                                   # the group is broken: no teardown


@pytest.mark.parametrize("mode", ["stays", "exits"])
def test_survivor_reports_a_rank_that_left_within_the_limit(mode):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_leaving_worker, args=(r, world, port, mode, q))
             for r in range(world)]
    for p in procs:
        p.start()
    kind, elapsed, detail = q.get(timeout=90)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert kind == "BackendError", (kind, detail)
    assert elapsed < LIMIT_S + 5.0, (elapsed, detail)
