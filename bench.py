"""Benchmark: HBM GB/s of rusttorch-core's hot path on B200 (BASELINE.json metric).

One step = one pass of the four ops the metric names, each on its
BASELINE.json config:
  add->mul_scalar  cfg1  2 x [2^24] U[-1,1)                 12 B/element
  sum              cfg2  [2^28] N(0,1)                        4 B/element
  softmax(dim=1)   cfg4  [32768, 4096] N(0,2)                 8 B/element
  adamw (in place) cfg5  4 x [2^30], lr 1e-3, b (0.9, 0.999),
                         eps 1e-8, wd 0.01, t 10             28 B/element
Strong scaling (default): on N GPUs rank r owns elements [r*n/N, (r+1)*n/N)
of cfg1, cfg2 and cfg5 and rows [r*32768/N, (r+1)*32768/N) of cfg4, cut from
the same seeded streams as the N = 1 tensors.  The sum's per-GPU f64
partials are all-reduced over peer memory (NVLink) by the library, the only
exchange (at the end of the step, after AdamW); the other ops need none.  `--scaling weak` gives every GPU a full-size copy instead.
value = algorithmic bytes of the whole step / max-over-ranks device time.

    python bench.py [--gpus N --steps K --warmup W] [--impl reference]
    torchrun --nproc-per-node N bench.py --gpus N ...
    python bench.py --suite [--only REGEX]     # every op alone, one GPU
    python bench.py --probe [--only REGEX]     # read/copy ceilings, cfg1 sizing

Prints ONE JSON line on rank 0 (one per op with --suite / --probe).
"""
from __future__ import annotations

import argparse
import ctypes
import json
import re
import os
import statistics
import subprocess
import sys
import time
from ctypes import byref, c_double, c_void_p
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "HBM GB/s (% of B200 peak) for add/sum/softmax/AdamW at 1/2/4/8 GPUs"
N1 = 1 << 24                       # cfg1
N2 = 1 << 28                       # cfg2
R3, C3 = 8192, 16384               # cfg3
R4, C4 = 32768, 4096               # cfg4
N5 = 1 << 30                       # cfg5
ADAMW = (1e-3, 0.9, 0.999, 1e-8, 0.01, 10)
BYTES = {
    "add_mul_scalar": 12 * N1,
    "sum": 4 * N2,
    "softmax": 8 * R4 * C4,
    "adamw": 28 * N5,
}
ELEMS = {"add_mul_scalar": N1, "sum": N2, "softmax": R4 * C4, "adamw": N5}
OPS = list(BYTES)
FALLBACK_HBM_GBS = 6650.0
SPEC_HBM_GBS = 8000.0              # B200 HBM3e data-sheet figure, for context


def peak_hbm() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    try:
        return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def env_int(k, d):
    try:
        return int(os.environ.get(k, d))
    except ValueError:
        return d


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """This GPU's SM clock and clock-event (throttle) reasons, sampled every
    few milliseconds during the timed region by a thread reading NVML (read
    only: nothing is set).  Falls back to `nvidia-smi -lms 50` if NVML is
    unavailable."""

    # nvmlClocksEventReasons bits
    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown",
               0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown"}
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, cuda_index: int, period_s: float = 0.005):
        self.cuda_index = cuda_index
        self.period = period_s
        self.samples = []          # (sm_mhz, max_mhz, reason_bits)
        self.proc = None
        self.thread = None
        self.path = Path(os.environ.get("TMPDIR", "/tmp")) / f"rt_clocks_{os.getpid()}.csv"

    def _handle(self, pynvml):
        try:
            import torch
            props = torch.cuda.get_device_properties(self.cuda_index)
            bus = f"{props.pci_domain_id:08x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
            return pynvml.nvmlDeviceGetHandleByPciBusId(bus)
        except Exception:
            return pynvml.nvmlDeviceGetHandleByIndex(self.cuda_index)

    def _sample(self):
        p = self.nvml
        sm = p.nvmlDeviceGetClockInfo(self.h, p.NVML_CLOCK_SM)
        try:
            bits = p.nvmlDeviceGetCurrentClocksEventReasons(self.h)
        except Exception:
            bits = p.nvmlDeviceGetCurrentClocksThrottleReasons(self.h)
        self.samples.append((sm, self.max_mhz, bits))

    def _loop(self):
        while not self.stop.is_set():
            try:
                self._sample()
            except Exception:
                return
            self.stop.wait(self.period)

    def __enter__(self):
        try:
            import threading
            import pynvml
            pynvml.nvmlInit()
            self.nvml = pynvml
            self.h = self._handle(pynvml)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self._sample()
            self.stop = threading.Event()
            self.thread = threading.Thread(target=self._loop, daemon=True)
            self.thread.start()
        except Exception:
            self.thread = None
            try:
                self.f = open(self.path, "w")
                self.proc = subprocess.Popen(
                    ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                     "-i", str(self.cuda_index), "-lms", "50"], stdout=self.f,
                    stderr=subprocess.DEVNULL)
            except Exception:
                self.proc = None
        return self

    def __exit__(self, *exc):
        if self.thread is not None:
            self.stop.set()
            self.thread.join(timeout=5)
            try:
                self._sample()
            except Exception:
                pass
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.f.close()

    def summary(self) -> dict:
        if self.samples:
            sm = [float(s[0]) for s in self.samples]
            reasons = sorted({name for _, _, bits in self.samples
                              for bit, name in self.REASONS.items() if bits & bit})
            return {"sm_mhz": statistics.median(sm), "sm_max_mhz": float(self.samples[0][1]),
                    "reasons": reasons, "samples": len(self.samples), "source": "nvml"}
        rows = []
        try:
            for line in self.path.read_text().splitlines():
                parts = [s.strip() for s in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        except Exception:
            pass
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        smax = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None, "reasons": reasons,
                "samples": len(rows), "source": "nvidia-smi"}


# ------------------------------------------------------------- CPU baseline
def cpu_step_sample(frac_log2: int = 6):
    """The reference's CPU path (oracle port) on 1/2^frac_log2 of every op's
    workload: returns a callable running one sampled step and its bytes."""
    from tests import _oracle as O

    s = 1 << frac_log2
    a, b = O.uniform(N1 // s, 1), O.uniform(N1 // s, 101)
    x2 = O.normal(N2 // s, 2)
    x4 = O.normal(R4 // s * C4, 4, 0.0, 2.0).reshape(R4 // s, C4)
    n5 = N5 // s
    p, g = O.normal(n5, 51, 0, 0.02), O.normal(n5, 52, 0, 1e-2)
    m, v = O.normal(n5, 53, 0, 1e-3), O.uniform(n5, 54, 0.0, 1e-4)
    total = sum(BYTES.values()) // s

    def step():
        c = O.binary("add", a, b)                    # rayon add (all cores)
        O.scalar_op("mul_scalar", c, 0.5)
        O.sum(x2)
        O.softmax(x4, 1)
        O.adamw(p, g, m, v, *ADAMW)

    return step, total, f"1/{s} of each op's workload (add {N1 // s}, sum {N2 // s}, softmax " \
                        f"{R4 // s}x{C4}, adamw {n5} elements)"


CPU_NOTE = ("conservative for the GPU: the C port runs 1/64 of each config (same byte mix) and "
            "fuses AdamW into one loop over the four buffers, where the reference makes about 13 "
            "allocating single-threaded ndarray passes (optimizer.rs:293-309, 413-421), so the "
            "reference itself would be slower than this figure")


def time_cpu(seconds_target: float = 12.0):
    from tests import _oracle as O

    step, nbytes, sample = cpu_step_sample()
    step()  # warm (page faults of first outputs)
    t0 = time.perf_counter()
    k = 0
    while True:
        step()
        k += 1
        el = time.perf_counter() - t0
        if el >= seconds_target or k >= 50:
            break
    return {"value": nbytes * k / el / 1e9, "unit": "GB/s", "cores": O.lib().rto_get_threads(),
            "kind": "port", "sample": sample + f"; {k} steps in {el:.1f} s; add runs on a "
            "thread per core (rayon in the reference), the other ops on one thread as ndarray "
            "does in the reference", "note": CPU_NOTE}


def run_reference(args) -> None:
    rank, world = env_int("RANK", 0), env_int("WORLD_SIZE", 1)
    if rank != 0:
        return
    from tests import _oracle as O

    step, nbytes, sample = cpu_step_sample()
    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    el = time.perf_counter() - t0
    value = nbytes * args.steps / el / 1e9
    cores = O.lib().rto_get_threads()
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "GB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": el / args.steps * 1e3, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded, BASELINE.json shapes)",
        "config": {"workload": "add->mul_scalar cfg1 + sum cfg2 + softmax cfg4 + adamw cfg5",
                   "sample": sample},
        "cpu_baseline": {"value": value, "unit": "GB/s", "cores": cores, "kind": "port",
                         "sample": sample, "note": CPU_NOTE},
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "rusttorch is Rust and no Rust toolchain exists here; the timed code is the C "
                "restatement of its CPU ops (oracle/), with its threading model",
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------- GPU arm
def shard_of(n: int, rank: int, world: int) -> tuple[int, int]:
    """Rank r's contiguous share [lo, hi) of n units (rows or elements)."""
    return n * rank // world, n * (rank + 1) // world


class Layout:
    """What one rank holds: under strong scaling its contiguous share of
    every config (cfg1/cfg2/cfg5 by elements, cfg4 by rows of 4096); under
    weak scaling a full-size shard of each (shard r = elements [r*n, (r+1)*n)
    of the same seeded stream).  `off*` are the offsets of the rank's first
    element in the global seeded stream, so the shards of all ranks together
    are exactly the N = 1 tensors."""

    def __init__(self, rank: int, world: int, scaling: str):
        self.scaling = scaling
        if scaling == "strong":
            lo1, hi1 = shard_of(N1, rank, world)
            lo2, hi2 = shard_of(N2, rank, world)
            lo4, hi4 = shard_of(R4, rank, world)
            lo5, hi5 = shard_of(N5, rank, world)
            self.n1, self.off1 = hi1 - lo1, lo1
            self.n2, self.off2 = hi2 - lo2, lo2
            self.r4, self.off4 = hi4 - lo4, lo4 * C4
            self.n5, self.off5 = hi5 - lo5, lo5
        else:
            self.n1, self.off1 = N1, rank * N1
            self.n2, self.off2 = N2, rank * N2
            self.r4, self.off4 = R4, rank * R4 * C4
            self.n5, self.off5 = N5, rank * N5
        self.bytes = {"add_mul_scalar": 12 * self.n1, "sum": 4 * self.n2,
                      "softmax": 8 * self.r4 * C4, "adamw": 28 * self.n5}
        self.elems = {"add_mul_scalar": self.n1, "sum": self.n2, "softmax": self.r4 * C4,
                      "adamw": self.n5}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--scaling", default="strong", choices=["strong", "weak"],
                    help="strong (default): the BASELINE configs split over the N GPUs; weak: "
                         "every GPU holds a full-size copy of each config")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--ops", default=",".join(OPS),
                    help="subset of ops in the step (profiling); the JSON line needs all four")
    ap.add_argument("--suite", action="store_true",
                    help="time every op of every config alone (L2 flushed between runs); "
                         "prints one JSON line per op")
    ap.add_argument("--only", default="",
                    help="with --suite: time only the ops whose name matches this regex")
    ap.add_argument("--configs", default="cfg1,cfg2,cfg3,cfg4,cfg5",
                    help="with --suite: the configs to allocate and time (profiling)")
    ap.add_argument("--small", action="store_true",
                    help="profiling case: sum 2^26, softmax 8192x4096, adamw 4x2^26 (all > L2)")
    args = ap.parse_args()
    if args.small:
        global N2, R3, R4, N5
        N2, R3, R4, N5 = 1 << 26, 2048, 8192, 1 << 26
        BYTES.update(sum=4 * N2, softmax=8 * R4 * C4, adamw=28 * N5)
        args.no_e2e = args.no_cpu_baseline = True
    if args.impl == "reference":
        run_reference(args)
        return
    args.warmup = max(args.warmup, 3)
    if args.suite:
        run_suite(args)
        return

    import torch
    import torch.distributed as dist

    from rusttorch_b200 import _native as N

    rank, world = env_int("RANK", 0), env_int("WORLD_SIZE", 1)
    local = env_int("LOCAL_RANK", 0)
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    L = Layout(rank, world, args.scaling)
    lib = N.lib()
    stream = torch.cuda.current_stream()
    N.check(lib.rtc_set_stream(c_void_p(stream.cuda_stream)))
    ops = [o for o in args.ops.split(",") if o]

    def empty(n):
        return torch.empty(max(n, 1), dtype=torch.float32, device="cuda")

    def desc(t, shape):
        return N.Desc(t.data_ptr(), shape, N.F32, local)

    def fill(t, shape, seed, normal, a_, b_, offset):
        fn = lib.rtc_fill_normal if normal else lib.rtc_fill_uniform
        N.check(fn(desc(t, shape).ref, seed, offset, a_, b_))

    shape = {"a": [L.n1], "b": [L.n1], "c": [L.n1], "x2": [L.n2], "x4": [L.r4, C4],
             "y4": [L.r4, C4], "p": [L.n5], "g": [L.n5], "m": [L.n5], "v": [L.n5]}
    bufs = {}
    if "add_mul_scalar" in ops:
        bufs["a"], bufs["b"], bufs["c"] = empty(L.n1), empty(L.n1), empty(L.n1)
        fill(bufs["a"], [L.n1], 1, False, -1.0, 1.0, L.off1)
        fill(bufs["b"], [L.n1], 101, False, -1.0, 1.0, L.off1)
    if "sum" in ops:
        bufs["x2"] = empty(L.n2)
        fill(bufs["x2"], [L.n2], 2, True, 0.0, 1.0, L.off2)
    if "softmax" in ops:
        bufs["x4"], bufs["y4"] = empty(L.r4 * C4), empty(L.r4 * C4)
        fill(bufs["x4"], [L.r4, C4], 4, True, 0.0, 2.0, L.off4)
    if "adamw" in ops:
        for k, seed, normal, a_, b_ in (("p", 51, True, 0.0, 0.02), ("g", 52, True, 0.0, 1e-2),
                                        ("m", 53, True, 0.0, 1e-3), ("v", 54, False, 0.0, 1e-4)):
            bufs[k] = empty(L.n5)
            fill(bufs[k], [L.n5], seed, normal, a_, b_, L.off5)
    D = {k: desc(bufs[k], shape[k]) for k in bufs}
    torch.cuda.synchronize()

    # Before timing (N > 1): the sharded sum/max/min of cfg2 through the
    # exact per-shard summaries, all-gathered and folded in rank order,
    # against the peer-memory all-reduce of the f64 partials the timed step
    # uses (and against NCCL's all-reduce of the same partials).
    check = None
    peer = None
    sum_dev = torch.zeros(1, dtype=torch.float64, device="cuda")
    sum_all = torch.zeros(1, dtype=torch.float64, device="cuda")
    if world > 1 and "sum" in ops:
        from rusttorch_b200 import sharded as sh
        exact = sh.ShardedReducer(lib, rank, world).stats(D["x2"])
        peer = sh.PeerSum(lib, rank, world, local)
        N.check(lib.rtc_sum_device(D["x2"].ref, c_void_p(sum_dev.data_ptr())))
        peer.allreduce(sum_dev.data_ptr(), sum_all.data_ptr())
        N.check(lib.rtc_synchronize())
        got = float(sum_all.item())
        nccl = sum_dev.clone()
        dist.all_reduce(nccl)
        absx = torch.tensor([float(bufs["x2"].abs().double().sum())], dtype=torch.float64,
                            device="cuda")
        dist.all_reduce(absx)
        tol = 1e-6 * float(absx.item())
        if abs(got - exact[0]) > tol:
            raise SystemExit(f"sharded sum mismatch: peer all-reduce {got!r} vs rank-order "
                             f"{exact[0]!r}")
        check = {"sum": exact[0], "mean": exact[1], "max": exact[2], "min": exact[3],
                 "allreduce_sum_minus_exact": got - exact[0],
                 "nccl_allreduce_sum_minus_exact": float(nccl.item()) - exact[0],
                 "tolerance": tol}

    # The sum lands in device memory without a host round trip; at N > 1 the
    # per-GPU f64 partials are combined (the hot path's only exchange) at the
    # end of the step, after AdamW, where every rank arrives after the same
    # work, by the library's peer-memory all-reduce (sharded.PeerSum: one
    # kernel per rank writes its partial into every rank's slots over NVLink
    # and adds the slots in rank order).  NCCL's all-reduce of the 8 bytes
    # cost 0.2-0.7 ms a step here, varying from run to run, at the end of the
    # step or on a second stream right after the sum (there it also waited
    # for the slowest rank's AdamW, whose grid holds every SM).
    def run_op(op):
        if op == "add_mul_scalar":
            N.check(lib.rtc_add_mul_scalar(D["a"].ref, D["b"].ref, 0.5, D["c"].ref))
        elif op == "sum":
            N.check(lib.rtc_sum_device(D["x2"].ref, c_void_p(sum_dev.data_ptr())))
        elif op == "softmax":
            N.check(lib.rtc_softmax(D["x4"].ref, 1, D["y4"].ref))
        elif op == "adamw":
            lr, b1, b2, eps, wd, t = ADAMW
            N.check(lib.rtc_adamw_update(D["p"].ref, D["g"].ref, D["m"].ref, D["v"].ref, lr, b1,
                                         b2, eps, wd, t, D["p"].ref, D["m"].ref, D["v"].ref))

    def combine(coll_ev=None):
        """The step's exchange: the sum's per-GPU partials all-reduced."""
        if peer is not None:
            if coll_ev is not None:
                coll_ev[0].record(stream)
            peer.allreduce(sum_dev.data_ptr(), sum_all.data_ptr())
            if coll_ev is not None:
                coll_ev[1].record(stream)

    def barrier():
        if world > 1:
            dist.barrier()

    for _ in range(args.warmup):
        for op in ops:
            run_op(op)
        combine()
    torch.cuda.synchronize()

    # Events around every op of every step; the ops' inputs are re-read only
    # a full step later, after >= 3.7 GB of other traffic per GPU (N <= 8),
    # so L2 (126 MB) holds none of them when they start.
    def evpair():
        return torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    ev = {op: [evpair() for _ in range(args.steps)] for op in ops}
    coll = [evpair() for _ in range(args.steps)]
    start, stop = evpair()
    barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clocks:
        if world > 1:
            # The GPU idles 20 ms (untimed) while this process queues all K
            # steps, so no step waits for the host (the clock sampler's
            # thread can hold Python's lock for milliseconds); then one
            # untimed exchange lines the ranks up, since they leave the
            # barrier above at different host times and every step's
            # exchange would otherwise absorb that skew.
            torch.cuda._sleep(40_000_000)
            combine()
        start.record(stream)
        for k in range(args.steps):
            for op in ops:
                e0, e1 = ev[op][k]
                e0.record(stream)
                run_op(op)
                e1.record(stream)
            combine(coll[k])
        stop.record(stream)
        torch.cuda.synchronize()
    barrier()
    total_ms = start.elapsed_time(stop)
    op_ms = {op: sum(e0.elapsed_time(e1) for e0, e1 in ev[op]) / args.steps for op in ops}
    coll_ms = (sum(e0.elapsed_time(e1) for e0, e1 in coll) / args.steps
               if world > 1 and "sum" in ops else 0.0)
    if world > 1:
        t = torch.tensor([total_ms, coll_ms] + [op_ms[o] for o in ops], dtype=torch.float64,
                         device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms, coll_ms = float(t[0]), float(t[1])
        op_ms = {o: float(t[i + 2]) for i, o in enumerate(ops)}
    ms_step = total_ms / args.steps
    rank_bytes = sum(L.bytes[o] for o in ops)
    step_bytes = rank_bytes * world if args.scaling == "weak" else sum(BYTES[o] for o in ops)
    value = step_bytes / (ms_step * 1e-3) / 1e9
    peak, peak_kind = peak_hbm()
    per_op = {o: {"ms": op_ms[o], "GB_s_per_gpu": L.bytes[o] / (op_ms[o] * 1e-3) / 1e9,
                  "elements_per_s_per_gpu": L.elems[o] / (op_ms[o] * 1e-3),
                  "frac_of_measured_peak": L.bytes[o] / (op_ms[o] * 1e-3) / 1e9 / peak,
                  "frac_of_8TBs_spec": L.bytes[o] / (op_ms[o] * 1e-3) / 1e9 / SPEC_HBM_GBS}
              for o in ops}
    if world > 1 and "sum" in ops:
        per_op["sum"]["peer_allreduce_ms"] = coll_ms
    dom = max(ops, key=lambda o: op_ms[o])
    achieved = L.bytes[dom] / (op_ms[dom] * 1e-3) / 1e9
    traffic = None
    tf = ROOT / "profiles" / "traffic_per_launch.txt"
    if tf.exists():
        for line in tf.read_text().splitlines():
            parts = line.split()
            if len(parts) >= 3 and parts[0] == dom:
                # bytes per element, from the ncu capture, times this launch's elements
                traffic = int(round(float(parts[2]) * L.elems[dom]))
    gpu_launches = args.steps * (sum({"add_mul_scalar": 1, "sum": 2, "softmax": 1,
                                      "adamw": 1}[o] for o in ops) + (peer is not None))

    # e2e: the same step through the C ABI from pinned host buffers.
    e2e = None
    if not args.no_e2e and set(ops) == set(OPS):
        e2e = run_e2e(args, lib, N, torch, L, bufs, shape, rank, world)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and set(ops) == set(OPS):
        try:
            cpu = time_cpu()
        except Exception as ex:  # the oracle is test infrastructure; say why it is absent
            cpu = {"value": None, "unit": "GB/s", "cores": 0, "kind": "port",
                   "sample": f"unavailable: {ex}"}

    if rank == 0:
        split = ("cfg1/cfg2/cfg5 split into N contiguous element ranges, cfg4 into N row blocks"
                 if args.scaling == "strong" else "every GPU holds a full-size copy of each config")
        line = {
            "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
            "higher_is_better": True, "scaling": args.scaling, "vs_baseline": None,
            "dtype": "f32",
            "data": "synthetic (seeded device generator, BASELINE.json shapes/distributions)",
            "config": {"workload": "add->mul_scalar cfg1 [2^24] + sum cfg2 [2^28] + softmax "
                                   "cfg4 [32768,4096] dim 1 + adamw cfg5 4x[2^30]"
                                   + (" per GPU" if args.scaling == "weak" else
                                      ", split over the GPUs"),
                       "ops": ops, "step_bytes": step_bytes, "per_gpu_bytes_per_step": rank_bytes,
                       "split": split,
                       "l2": "no flush: each op's inputs are re-read only after >= 3.7 GB of "
                             "other traffic per GPU (L2 is 126 MB)",
                       "parallelism": f"dp{world} ({args.scaling})"},
            "frac_of_peak": value / (peak * world),
            "per_op": per_op,
            "roofline": {"bound": "hbm", "kernel": dom, "achieved": achieved, "peak": peak,
                         "unit": "GB/s", "frac": achieved / peak, "traffic": traffic,
                         "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)"
                         if peak_kind == "measured" else "fallback 6.65 TB/s"},
            "clocks": clocks.summary(),
            "gpu_launches": gpu_launches,
            "e2e": e2e,
            "cpu_baseline": cpu,
        }
        if check is not None:
            line["sharded_check"] = check
        print(json.dumps(line), flush=True)
    if peer is not None:
        peer.close()
    if world > 1:
        dist.destroy_process_group()


def run_e2e(args, lib, N, torch, L, bufs, shape, rank, world):
    """The same step through the C ABI on tensors in pinned host memory
    (rtc_tensor.device = RTC_HOST_MEMORY): the library streams every op's
    inputs to the GPU and its results back (c, the sum, y, and p/m/v in
    place), copies overlapped with the kernels.  Each rank streams its own
    shard through its own GPU; at N > 1 the sum's shard summaries are
    all-gathered and folded in rank order.  Timed on the host clock from the
    first input byte to the last result byte, max over ranks."""
    import torch.distributed as dist

    k_e2e = max(1, min(args.steps, 3))
    HOST = -1
    host = {}
    for k in ("a", "b", "c", "x2", "x4", "y4", "p", "g", "m", "v"):
        host[k] = torch.empty(bufs[k].numel(), dtype=torch.float32, pin_memory=True)
        host[k].copy_(bufs[k])
    torch.cuda.synchronize()
    H = {k: N.Desc(host[k].data_ptr(), shape[k], N.F32, HOST) for k in host}
    h2d = sum(host[k].numel() * 4 for k in ("a", "b", "x2", "x4", "p", "g", "m", "v"))
    d2h = sum(host[k].numel() * 4 for k in ("c", "y4", "p", "m", "v"))
    lr, b1, b2, eps, wd, t = ADAMW
    reducer = None
    if world > 1:
        from rusttorch_b200 import sharded as sh
        reducer = sh.ShardedReducer(lib, rank, world)
    out = c_double()

    def step():
        N.check(lib.rtc_add_mul_scalar(H["a"].ref, H["b"].ref, 0.5, H["c"].ref))
        if reducer is None:
            N.check(lib.rtc_sum(H["x2"].ref, byref(out)))
        else:
            out.value = reducer.stats(H["x2"])[0]
        N.check(lib.rtc_softmax(H["x4"].ref, 1, H["y4"].ref))
        N.check(lib.rtc_adamw_update(H["p"].ref, H["g"].ref, H["m"].ref, H["v"].ref, lr, b1, b2,
                                     eps, wd, t, H["p"].ref, H["m"].ref, H["v"].ref))

    step()
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(k_e2e):
        step()
    ms = (time.perf_counter() - t0) * 1e3 / k_e2e
    if world > 1:
        tt = torch.tensor([ms], dtype=torch.float64, device="cuda")
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms = float(tt[0])
    total = sum(L.bytes.values()) * (world if L.scaling == "weak" else 1)
    if L.scaling == "strong":
        total = sum(BYTES.values())
    value = total / (ms * 1e-3) / 1e9
    return {"value": value, "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "ms_per_step": ms, "steps": k_e2e,
            "path": "C-ABI ops on pinned host tensors (device = RTC_HOST_MEMORY): chunked H2D, "
                    "kernel and D2H overlapped on three streams inside the library; each rank "
                    "streams its own shard"}


def run_suite(args) -> None:
    """Every op of every BASELINE.json config, timed alone on one GPU: CUDA
    events around each call, L2 flushed (256 MiB written, 256 MiB read)
    before each one,
    median of max(3, --steps) runs.  One JSON line per op."""
    import torch

    from rusttorch_b200 import _native as N

    torch.cuda.set_device(0)
    lib = N.lib()
    stream = torch.cuda.current_stream()
    N.check(lib.rtc_set_stream(c_void_p(stream.cuda_stream)))
    peak, _ = peak_hbm()
    # L2 flush before each run: 256 MiB written, then another 256 MiB read,
    # so the run starts with no line of its inputs in L2 and no dirty line
    # left to write back (the write alone would leave an L2 of dirty lines
    # for the timed kernel to evict: 7 % of a 201 MB op, see --probe).
    flush = torch.empty(64 << 20, dtype=torch.float32, device="cuda")
    flush_rd = torch.ones(64 << 20, dtype=torch.float32, device="cuda")

    def t(shape):
        n = 1
        for d in shape:
            n *= d
        x = torch.empty(n, dtype=torch.float32, device="cuda")
        return x, N.Desc(x.data_ptr(), shape, N.F32, 0)

    def fill(pair, seed, normal=False, a=-1.0, b=1.0):
        fn = lib.rtc_fill_normal if normal else lib.rtc_fill_uniform
        N.check(fn(pair[1].ref, seed, 0, a, b))

    only = re.compile(args.only) if args.only else None

    def timeit(name, cfg, nbytes, fn, elems=None):
        if only is not None and not only.search(name):
            return
        for _ in range(2):
            fn()
        times = []
        for _ in range(max(3, args.steps)):
            flush.zero_()
            flush_rd.sum()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            fn()
            e1.record(stream)
            torch.cuda.synchronize()
            times.append(e0.elapsed_time(e1))
        ms = statistics.median(times)
        gbs = nbytes / (ms * 1e-3) / 1e9
        row = {"op": name, "config": cfg, "ms": ms, "GB_s": gbs,
               "frac_of_measured_peak": gbs / peak, "frac_of_8TBs_spec": gbs / SPEC_HBM_GBS,
               "bytes": nbytes}
        if elems is None:
            elems = {"cfg1": N1, "cfg2": N2, "cfg3": R3 * C3, "cfg4": R4 * C4,
                     "cfg5": N5}.get(cfg[:4])
        if elems:
            row["elements_per_s"] = elems / (ms * 1e-3)
        print(json.dumps(row), flush=True)

    lr, b1, b2, eps, wd, tt = ADAMW
    cfgs = set(args.configs.split(","))
    if "cfg1" in cfgs:   # cfg1
        a, b, c = t([N1]), t([N1]), t([N1])
        fill(a, 1)
        fill(b, 101)
        for name, fn in (("add", lib.rtc_add), ("sub", lib.rtc_sub), ("mul", lib.rtc_mul),
                         ("div", lib.rtc_div)):
            timeit(name, f"cfg1 [{N1}]", 12 * N1,
                   lambda fn=fn: N.check(fn(a[1].ref, b[1].ref, c[1].ref)))
        timeit("mul_scalar", f"cfg1 [{N1}]", 8 * N1,
               lambda: N.check(lib.rtc_mul_scalar(a[1].ref, 0.5, c[1].ref)))
        timeit("add->mul_scalar (fused)", f"cfg1 [{N1}]", 12 * N1,
               lambda: N.check(lib.rtc_add_mul_scalar(a[1].ref, b[1].ref, 0.5, c[1].ref)))
        timeit("add then mul_scalar (two kernels)", f"cfg1 [{N1}]", 20 * N1,
               lambda: (N.check(lib.rtc_add(a[1].ref, b[1].ref, c[1].ref)),
                        N.check(lib.rtc_mul_scalar(c[1].ref, 0.5, c[1].ref))))
        # losses (ops/loss.rs) on cfg1's shape: predictions uniform in [0, 1);
        # targets uniform in [-1, 1) for the regression losses and in [0, 1) (soft
        # labels, the cross-entropies' domain) for bce/ce
        v1 = c_double()
        fill(c, 102, False, 0.0, 1.0)
        fill(b, 103, False, 0.0, 1.0)
        for name, fn, extra, tg in (("mse_loss", lib.rtc_mse_loss, (), a),
                                    ("l1_loss", lib.rtc_l1_loss, (), a),
                                    ("smooth_l1_loss", lib.rtc_smooth_l1_loss, (1.0,), a),
                                    ("binary_cross_entropy_loss", lib.rtc_binary_cross_entropy_loss,
                                     (1e-7,), b),
                                    ("cross_entropy_loss", lib.rtc_cross_entropy_loss, (1e-7,), b)):
            timeit(name, f"cfg1 [{N1}]", 8 * N1,
                   lambda fn=fn, extra=extra, tg=tg: N.check(fn(c[1].ref, tg[1].ref, *extra,
                                                                byref(v1))))
        del a, b, c
    if "cfg2" in cfgs:   # cfg2
        x = t([N2])
        fill(x, 2, True, 0.0, 1.0)
        sd = torch.zeros(1, dtype=torch.float64, device="cuda")
        v = c_double()
        timeit("sum (device result)", f"cfg2 [{N2}]", 4 * N2,
               lambda: N.check(lib.rtc_sum_device(x[1].ref, c_void_p(sd.data_ptr()))))
        for name, fn in (("sum", lib.rtc_sum), ("mean", lib.rtc_mean), ("max", lib.rtc_max),
                         ("min", lib.rtc_min)):
            timeit(name + " (host result)", f"cfg2 [{N2}]", 4 * N2,
                   lambda fn=fn: N.check(fn(x[1].ref, byref(v))))
        st4 = (c_double * 4)()
        timeit("stats: sum+mean+max+min, one pass (host result)", f"cfg2 [{N2}]", 4 * N2,
               lambda: N.check(lib.rtc_stats(x[1].ref, st4)))
        del x
    if "cfg3" in cfgs:   # cfg3
        x = t([R3, C3])
        fill(x, 3)
        for dim, outn in ((1, R3), (0, C3)):
            o = t([outn])
            for name, fn in (("sum_dim", lib.rtc_sum_dim), ("mean_dim", lib.rtc_mean_dim),
                             ("max_dim", lib.rtc_max_dim)):
                timeit(f"{name}({dim})", f"cfg3 [{R3},{C3}]", 4 * R3 * C3 + 4 * outn,
                       lambda fn=fn, o=o, dim=dim: N.check(fn(x[1].ref, dim, o[1].ref)))
        del x
    if "cfg4" in cfgs:   # cfg4
        x, y = t([R4, C4]), t([R4, C4])
        fill(x, 4, True, 0.0, 2.0)
        for name in ("relu", "gelu", "swish", "sigmoid", "tanh", "selu", "softsign", "mish",
                     "softplus"):
            fn = getattr(lib, "rtc_" + name)
            timeit(name, f"cfg4 [{R4},{C4}]", 8 * R4 * C4,
                   lambda fn=fn: N.check(fn(x[1].ref, y[1].ref)))
        timeit("leaky_relu", f"cfg4 [{R4},{C4}]", 8 * R4 * C4,
               lambda: N.check(lib.rtc_leaky_relu(x[1].ref, y[1].ref, 0.01)))
        timeit("elu", f"cfg4 [{R4},{C4}]", 8 * R4 * C4,
               lambda: N.check(lib.rtc_elu(x[1].ref, y[1].ref, 1.0)))
        timeit("softmax(1)", f"cfg4 [{R4},{C4}]", 8 * R4 * C4,
               lambda: N.check(lib.rtc_softmax(x[1].ref, 1, y[1].ref)))
        bias = t([C4])
        fill(bias, 9)
        timeit("add_broadcast (row bias)", f"cfg4 [{R4},{C4}] + [{C4}]", 8 * R4 * C4 + 4 * C4,
               lambda: N.check(lib.rtc_add_broadcast(x[1].ref, bias[1].ref, y[1].ref)))
        # autograd backward (autograd/ops.rs) on cfg4's shape
        g, z, w = t([R4, C4]), t([R4, C4]), t([R4, C4])
        fill(g, 10, True, 0.0, 1.0)
        fill(z, 11, True, 1.0, 0.5)
        for name in ("relu", "sigmoid", "tanh", "gelu"):
            fn = getattr(lib, f"rtc_{name}_backward")
            timeit(f"{name}_backward", f"cfg4 [{R4},{C4}]", 12 * R4 * C4,
                   lambda fn=fn: N.check(fn(g[1].ref, x[1].ref, y[1].ref)))
        for name in ("mul", "div"):
            fn = getattr(lib, f"rtc_{name}_backward")
            timeit(f"{name}_backward (both grads)", f"cfg4 [{R4},{C4}]", 20 * R4 * C4,
                   lambda fn=fn: N.check(fn(g[1].ref, x[1].ref, z[1].ref, y[1].ref, w[1].ref)))
        cols, rows = t([1, C4]), t([R4, 1])
        timeit("broadcast_add_backward -> [1,C]", f"cfg4 [{R4},{C4}]", 4 * R4 * C4 + 4 * C4,
               lambda: N.check(lib.rtc_broadcast_add_backward(g[1].ref, cols[1].ref, None)))
        timeit("broadcast_add_backward -> [R,1]", f"cfg4 [{R4},{C4}]", 4 * R4 * C4 + 4 * R4,
               lambda: N.check(lib.rtc_broadcast_add_backward(g[1].ref, rows[1].ref, None)))
        del x, y, g, z, w
    if "cfg5" in cfgs:   # cfg5
        P = {k: t([N5]) for k in "pgmv"}
        fill(P["p"], 51, True, 0.0, 0.02)
        fill(P["g"], 52, True, 0.0, 1e-2)
        fill(P["m"], 53, True, 0.0, 1e-3)
        fill(P["v"], 54, False, 0.0, 1e-4)
        timeit("adamw (in place)", f"cfg5 4x[{N5}]", 28 * N5,
               lambda: N.check(lib.rtc_adamw_update(P["p"][1].ref, P["g"][1].ref, P["m"][1].ref,
                                                    P["v"][1].ref, lr, b1, b2, eps, wd, tt,
                                                    P["p"][1].ref, P["m"][1].ref, P["v"][1].ref)))

def run_probe(args) -> None:
    """Bandwidth probes (rtc_probe_stream): 1 GiB read with 16-byte loads
    and through a cp.async.bulk ring, a 1 GiB copy, and sizings of cfg1's
    fused add->mul_scalar map.  L2 flushed before each run, median of
    max(5, --steps) runs; one JSON line per configuration."""
    import torch

    from rusttorch_b200 import _native as N

    torch.cuda.set_device(0)
    lib = N.lib()
    stream = torch.cuda.current_stream()
    N.check(lib.rtc_set_stream(c_void_p(stream.cuda_stream)))
    peak, _ = peak_hbm()
    flush = torch.empty(64 << 20, dtype=torch.float32, device="cuda")
    flush_rd = torch.ones(64 << 20, dtype=torch.float32, device="cuda")
    nbytes = 1 << 30
    src = torch.randn(nbytes // 4, dtype=torch.float32, device="cuda")
    dst = torch.empty_like(src)
    only = re.compile(args.only) if args.only else None

    def lanes_match(p0, nb):
        """The lane-sum probe's output (dst) against the library's sum_dim(1)
        of the same [nb/4/p0, p0] view, bit for bit."""
        lanes = (nb // 4) // p0
        xs = N.Desc(src.data_ptr(), [lanes, p0], N.F32, 0)
        ref = torch.empty(lanes, dtype=torch.float32, device="cuda")
        N.check(lib.rtc_sum_dim(xs.ref, 1, N.Desc(ref.data_ptr(), [lanes], N.F32, 0).ref))
        torch.cuda.synchronize()
        return bool(torch.equal(ref.view(torch.int32), dst[:lanes].view(torch.int32)))

    def cols_match(p0, nb):
        """The strip probe's output (dst) against the library's sum_dim(0) of
        the same [nb/4/p0, p0] view, bit for bit."""
        rows = (nb // 4) // p0
        xs = N.Desc(src.data_ptr(), [rows, p0], N.F32, 0)
        ref = torch.empty(p0, dtype=torch.float32, device="cuda")
        N.check(lib.rtc_sum_dim(xs.ref, 0, N.Desc(ref.data_ptr(), [p0], N.F32, 0).ref))
        torch.cuda.synchronize()
        return bool(torch.equal(ref.view(torch.int32), dst[:p0].view(torch.int32)))

    def timeit(name, mode, nb, algo_bytes, p0, p1, p2, dirty=False):
        """dirty=False: L2 flushed by writing 256 MiB and then reading another
        256 MiB, so the timed kernel starts on clean lines; dirty=True: the
        write alone, so the kernel also writes back up to an L2 of dirty lines."""
        if only is not None and not only.search(name):
            return
        call = lambda: N.check(lib.rtc_probe_stream(mode, c_void_p(src.data_ptr()),
                                                    c_void_p(dst.data_ptr()), nb, p0, p1, p2))
        for _ in range(2):
            call()
        times = []
        for _ in range(max(5, args.steps)):
            flush.zero_()
            if not dirty:
                flush_rd.sum()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(args.repeat):
                call()
            e1.record(stream)
            torch.cuda.synchronize()
            times.append(e0.elapsed_time(e1) / args.repeat)
        N.check(lib.rtc_synchronize())
        ms = statistics.median(times)
        gbs = algo_bytes / (ms * 1e-3) / 1e9
        line = {"probe": name, "mode": mode, "p": [p0, p1, p2], "ms": ms, "GB_s": gbs,
                "frac_of_measured_peak": gbs / peak, "bytes": algo_bytes,
                "l2": "dirty" if dirty else "clean", "repeat": args.repeat}
        if mode == 8:
            line["matches_sum_dim"] = lanes_match(p0, nb)
        if mode == 9:
            line["matches_sum_dim"] = cols_match(p0, nb)
        print(json.dumps(line), flush=True)

    # u < 0: the stats kernel with float32 trees per float4 (|u| loads in flight)
    for threads, u, bps in ((256, 8, 0), (512, 4, 0), (512, 8, 0), (256, -4, 0), (256, -8, 0),
                            (512, -4, 0), (512, -8, 0), (1024, -4, 0), (512, -8, 2),
                            (256, -8, 4), (256, -8, 6), (-512, -8, 0), (-512, 8, 0),
                            (256, 2, 100), (256, 4, 100), (512, 2, 100), (512, 4, 100),
                            (512, 2, 104), (256, 4, 108)):
        timeit(f"stats kernel t{threads} u{u} b{bps}", 7, nbytes, nbytes, threads, u, bps)
    # cfg3's sum_dim(1): [8192, 16384]; negative: the direct-chain kernel,
    # -(1000*CPT + 10*K + warps per CTA), CPT chains per thread; >= 100: the
    # 128-byte-read transpose kernel, 100*K + warps per CTA
    for warps in (-2322, 802, 804, 808, 1202, 1204, 1602, 1604, 1608):
        timeit(f"lane sum [8192,16384] warps/CTA {warps}", 8, 4 * R3 * C3, 4 * R3 * C3 + 4 * R3,
               C3, warps, 0)
    # cfg4's broadcast_add_backward onto [1, C]: a dim-0 sum of [32768, 4096];
    # p1 columns per CTA, p2 = 100 * rows per tile + ring stages
    # (W >= 1000: the run-time-width kernel for W - 1000 columns)
    for w, code in ((1016, 25606), (16, 25606), (32, 25606), (1032, 25606), (32, 12808),
                    (16, 12808), (8, 25608), (4, 25608), (64, 12806)):
        timeit(f"strip dim0 [{R4},{C4}] W{w} p{code}", 9, 4 * R4 * C4, 4 * R4 * C4 + 4 * C4,
               C4, w, code)
    for dirty in (False, True):
        tag = "dirty-L2" if dirty else "clean-L2"
        timeit(f"{tag} cfg1 add->mul_scalar product", 5, 8 * N1, 12 * N1, 0, 4, 32, dirty)
        timeit(f"{tag} read ldg t512 u4 b4", 0, nbytes, nbytes, 512, 4, 4, dirty)
        timeit(f"{tag} copy ldg/stg t256 u8 b8", 4, nbytes, 2 * nbytes, 256, 8, 8, dirty)
    for threads in (256, 512, 1024):
        for u in (4, 8, 16):
            for bps in (1, 2, 4, 8):
                if threads * bps > 2048:
                    continue
                timeit(f"read ldg grid-stride t{threads} u{u} b{bps}", 0, nbytes, nbytes,
                       threads, u, bps)
                timeit(f"read ldg contiguous t{threads} u{u} b{bps}", 1, nbytes, nbytes,
                       threads, u, bps)
    for chunk in (4096, 8192, 16384, 32768):
        for slots in (2, 4, 6, 8, 12, 16):
            for ctas in (1, 2, 4):
                if chunk * slots * ctas > 200 * 1024 or chunk * slots > 200 * 1024:
                    continue
                if chunk * slots * ctas < 32 * 1024:
                    continue
                timeit(f"read bulk ring c{chunk} s{slots} x{ctas}", 2, nbytes, nbytes,
                       chunk, slots, ctas)
                timeit(f"read bulk ring+fold c{chunk} s{slots} x{ctas}", 3, nbytes, nbytes,
                       chunk, slots, ctas)
    for u in (4, 8):
        for bps in (4, 8):
            timeit(f"copy ldg/stg t256 u{u} b{bps}", 4, nbytes, 2 * nbytes, 256, u, bps)
    n1 = N1
    for mode, label in ((5, "grid-stride"), (6, "balanced")):
        for u in (1, 2, 4, 8):
            for bps in ((-1, 0, 2, 4, 8, 16, 32, 64) if mode == 5 else (0, 1, 2, 4, 8, 16)):
                timeit(f"cfg1 add->mul_scalar {label} u{u} b{bps}", mode, 8 * n1, 12 * n1,
                       0, u, bps)


if __name__ == "__main__":
    if "--probe" in sys.argv:
        ap = argparse.ArgumentParser()
        ap.add_argument("--probe", action="store_true")
        ap.add_argument("--steps", type=int, default=9)
        ap.add_argument("--only", default="")
        ap.add_argument("--repeat", type=int, default=1,
                        help="calls back to back between the events (launch gaps hidden)")
        run_probe(ap.parse_args())
    else:
        main()
