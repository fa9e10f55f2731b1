"""Benchmark: HBM GB/s of rusttorch-core's hot path on B200 (BASELINE.json metric).

One step = one pass of the four ops the metric names, each on its
BASELINE.json config, per GPU (weak scaling: every rank owns one full-size
shard of each tensor; shard r holds elements [r*n, (r+1)*n) of one seeded
global stream):
  add->mul_scalar  cfg1  2 x [2^24] U[-1,1)                 12 B/element
  sum              cfg2  [2^28] N(0,1); N > 1: local exact   4 B/element
                         summary + NCCL all-gather + rank-order combine
  softmax(dim=1)   cfg4  [32768, 4096] N(0,2)                 8 B/element
  adamw (in place) cfg5  4 x [2^30], lr 1e-3, b (0.9, 0.999),
                         eps 1e-8, wd 0.01, t 10             28 B/element
value = algorithmic bytes of all ranks / max-over-ranks device time.

    python bench.py [--gpus N --steps K --warmup W] [--impl reference]
    torchrun --nproc-per-node N bench.py --gpus N ...

Prints ONE JSON line on rank 0.
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
            "does in the reference"}


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
                         "sample": sample},
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "rusttorch is Rust and no Rust toolchain exists here; the timed code is the C "
                "restatement of its CPU ops (oracle/), with its threading model",
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------- GPU arm
def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--ops", default=",".join(OPS),
                    help="subset of ops in the step (profiling); the JSON line needs all four")
    ap.add_argument("--suite", action="store_true",
                    help="time every op of every config alone (L2 flushed between runs); "
                         "prints one JSON line per op")
    ap.add_argument("--only", default="",
                    help="with --suite: time only the ops whose name matches this regex")
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

    import rusttorch_b200 as rt
    from rusttorch_b200 import _native as N

    rank, world = env_int("RANK", 0), env_int("WORLD_SIZE", 1)
    local = env_int("LOCAL_RANK", 0)
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=180),
                                device_id=torch.device("cuda", local))
    lib = N.lib()
    stream = torch.cuda.current_stream()
    N.check(lib.rtc_set_stream(c_void_p(stream.cuda_stream)))
    ops = [o for o in args.ops.split(",") if o]

    def empty(n):
        return torch.empty(n, dtype=torch.float32, device="cuda")

    def desc(t, shape):
        return N.Desc(t.data_ptr(), shape, N.F32, local)

    def fill(t, shape, seed, normal, a_, b_):
        d = desc(t, shape)
        n = t.numel()
        fn = lib.rtc_fill_normal if normal else lib.rtc_fill_uniform
        N.check(fn(d.ref, seed, rank * n, a_, b_))

    bufs = {}
    if "add_mul_scalar" in ops:
        bufs["a"], bufs["b"], bufs["c"] = empty(N1), empty(N1), empty(N1)
        fill(bufs["a"], [N1], 1, False, -1.0, 1.0)
        fill(bufs["b"], [N1], 101, False, -1.0, 1.0)
    if "sum" in ops:
        bufs["x2"] = empty(N2)
        fill(bufs["x2"], [N2], 2, True, 0.0, 1.0)
    if "softmax" in ops:
        bufs["x4"], bufs["y4"] = empty(R4 * C4), empty(R4 * C4)
        fill(bufs["x4"], [R4, C4], 4, True, 0.0, 2.0)
    if "adamw" in ops:
        for k, seed, normal, a_, b_ in (("p", 51, True, 0.0, 0.02), ("g", 52, True, 0.0, 1e-2),
                                        ("m", 53, True, 0.0, 1e-3), ("v", 54, False, 0.0, 1e-4)):
            bufs[k] = empty(N5)
            fill(bufs[k], [N5], seed, normal, a_, b_)
    D = {}
    if "add_mul_scalar" in ops:
        D["a"], D["b"], D["c"] = (desc(bufs[k], [N1]) for k in "abc")
    if "sum" in ops:
        D["x2"] = desc(bufs["x2"], [N2])
    if "softmax" in ops:
        D["x4"], D["y4"] = desc(bufs["x4"], [R4, C4]), desc(bufs["y4"], [R4, C4])
    if "adamw" in ops:
        for k in "pgmv":
            D[k] = desc(bufs[k], [N5])
    torch.cuda.synchronize()

    # The sum lands in device memory without a host round trip; at N > 1 the
    # f64 partials are all-gathered over NCCL (the hot path's only exchange).
    sum_dev = torch.zeros(1, dtype=torch.float64, device="cuda")
    sum_all = torch.zeros(world, dtype=torch.float64, device="cuda")

    def run_op(op):
        if op == "add_mul_scalar":
            N.check(lib.rtc_add_mul_scalar(D["a"].ref, D["b"].ref, 0.5, D["c"].ref))
        elif op == "sum":
            N.check(lib.rtc_sum_device(D["x2"].ref, c_void_p(sum_dev.data_ptr())))
            if world > 1:
                dist.all_gather_into_tensor(sum_all, sum_dev)
        elif op == "softmax":
            N.check(lib.rtc_softmax(D["x4"].ref, 1, D["y4"].ref))
        elif op == "adamw":
            lr, b1, b2, eps, wd, t = ADAMW
            N.check(lib.rtc_adamw_update(D["p"].ref, D["g"].ref, D["m"].ref, D["v"].ref, lr, b1,
                                         b2, eps, wd, t, D["p"].ref, D["m"].ref, D["v"].ref))

    def barrier():
        if world > 1:
            dist.barrier()

    for _ in range(args.warmup):
        for op in ops:
            run_op(op)
    torch.cuda.synchronize()

    # Events around every op of every step; the ops' inputs are re-read only
    # a full step later, after >= 17 GB of other traffic, so L2 (126 MB) holds
    # none of them when they start.
    ev = {op: [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(args.steps)] for op in ops}
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clocks:
        start.record(stream)
        for k in range(args.steps):
            for op in ops:
                e0, e1 = ev[op][k]
                e0.record(stream)
                run_op(op)
                e1.record(stream)
        stop.record(stream)
        torch.cuda.synchronize()
    barrier()
    total_ms = start.elapsed_time(stop)
    op_ms = {op: sum(e0.elapsed_time(e1) for e0, e1 in ev[op]) / args.steps for op in ops}
    if world > 1:
        t = torch.tensor([total_ms] + [op_ms[o] for o in ops], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        total_ms = float(t[0])
        op_ms = {o: float(t[i + 1]) for i, o in enumerate(ops)}
    ms_step = total_ms / args.steps
    step_bytes = sum(BYTES[o] for o in ops) * world
    value = step_bytes / (ms_step * 1e-3) / 1e9
    peak, peak_kind = peak_hbm()
    per_op = {o: {"ms": op_ms[o], "GB_s": BYTES[o] / (op_ms[o] * 1e-3) / 1e9,
                  "elements_per_s": ELEMS[o] / (op_ms[o] * 1e-3),
                  "frac_of_measured_peak": BYTES[o] / (op_ms[o] * 1e-3) / 1e9 / peak,
                  "frac_of_8TBs_spec": BYTES[o] / (op_ms[o] * 1e-3) / 1e9 / SPEC_HBM_GBS}
              for o in ops}
    dom = max(ops, key=lambda o: op_ms[o])
    achieved = BYTES[dom] / (op_ms[dom] * 1e-3) / 1e9
    traffic = None
    tf = ROOT / "profiles" / "traffic_per_launch.txt"
    if tf.exists():
        for line in tf.read_text().splitlines():
            parts = line.split()
            if len(parts) >= 2 and parts[0] == dom:
                traffic = int(parts[1])
    gpu_launches = args.steps * sum({"add_mul_scalar": 1, "sum": 2, "softmax": 1,
                                     "adamw": 1}[o] for o in ops)

    # e2e: the same step through the C ABI from pinned host buffers.
    e2e = None
    if not args.no_e2e and set(ops) == set(OPS):
        e2e = run_e2e(args, lib, N, torch, D, bufs, rank, world, stream)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline and set(ops) == set(OPS):
        try:
            cpu = time_cpu()
        except Exception as ex:  # the oracle is test infrastructure; say why it is absent
            cpu = {"value": None, "unit": "GB/s", "cores": 0, "kind": "port",
                   "sample": f"unavailable: {ex}"}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_step,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded device generator, BASELINE.json shapes/distributions)",
            "config": {"workload": "add->mul_scalar cfg1 [2^24] + sum cfg2 [2^28] + softmax "
                                   "cfg4 [32768,4096] dim 1 + adamw cfg5 4x[2^30] per GPU",
                       "ops": ops, "per_gpu_bytes_per_step": step_bytes // world,
                       "l2": "no flush: each op's inputs are re-read only after >= 17 GB of "
                             "other traffic (L2 is 126 MB)",
                       "parallelism": f"dp{world} (weak: one full shard per GPU)"},
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
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def run_e2e(args, lib, N, torch, D, bufs, rank, world, stream):
    """The same step through the C ABI on tensors in pinned host memory
    (rtc_tensor.device = RTC_HOST_MEMORY): the library streams every op's
    inputs to the GPU and its results back (c, the sum, y, and p/m/v in
    place), copies overlapped with the kernels.  Timed on the host clock
    from the first input byte to the last result byte, max over ranks."""
    import torch.distributed as dist

    k_e2e = max(1, min(args.steps, 3))
    HOST = -1
    host = {}
    for k in ("a", "b", "c", "x2", "x4", "y4", "p", "g", "m", "v"):
        host[k] = torch.empty(bufs[k].numel(), dtype=torch.float32, pin_memory=True)
        host[k].copy_(bufs[k])
    torch.cuda.synchronize()
    shape = {"a": [N1], "b": [N1], "c": [N1], "x2": [N2], "x4": [R4, C4], "y4": [R4, C4],
             "p": [N5], "g": [N5], "m": [N5], "v": [N5]}
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
    value = sum(BYTES.values()) * world / (ms * 1e-3) / 1e9
    return {"value": value, "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "ms_per_step": ms, "steps": k_e2e,
            "path": "C-ABI ops on pinned host tensors (device = RTC_HOST_MEMORY): chunked H2D, "
                    "kernel and D2H overlapped on three streams inside the library"}


def run_suite(args) -> None:
    """Every op of every BASELINE.json config, timed alone on one GPU: CUDA
    events around each call, L2 flushed (256 MiB written) before each one,
    median of max(3, --steps) runs.  One JSON line per op."""
    import torch

    from rusttorch_b200 import _native as N

    torch.cuda.set_device(0)
    lib = N.lib()
    stream = torch.cuda.current_stream()
    N.check(lib.rtc_set_stream(c_void_p(stream.cuda_stream)))
    peak, _ = peak_hbm()
    flush = torch.empty(64 << 20, dtype=torch.float32, device="cuda")

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
    # cfg1
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
    # cfg2
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
    # cfg3
    x = t([R3, C3])
    fill(x, 3)
    for dim, outn in ((1, R3), (0, C3)):
        o = t([outn])
        for name, fn in (("sum_dim", lib.rtc_sum_dim), ("mean_dim", lib.rtc_mean_dim),
                         ("max_dim", lib.rtc_max_dim)):
            timeit(f"{name}({dim})", f"cfg3 [{R3},{C3}]", 4 * R3 * C3 + 4 * outn,
                   lambda fn=fn, o=o, dim=dim: N.check(fn(x[1].ref, dim, o[1].ref)))
    del x
    # cfg4
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
    # cfg5
    P = {k: t([N5]) for k in "pgmv"}
    fill(P["p"], 51, True, 0.0, 0.02)
    fill(P["g"], 52, True, 0.0, 1e-2)
    fill(P["m"], 53, True, 0.0, 1e-3)
    fill(P["v"], 54, False, 0.0, 1e-4)
    timeit("adamw (in place)", f"cfg5 4x[{N5}]", 28 * N5,
           lambda: N.check(lib.rtc_adamw_update(P["p"][1].ref, P["g"][1].ref, P["m"][1].ref,
                                                P["v"][1].ref, lr, b1, b2, eps, wd, tt,
                                                P["p"][1].ref, P["m"][1].ref, P["v"][1].ref)))


if __name__ == "__main__":
    main()
