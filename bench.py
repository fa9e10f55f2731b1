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
R4, C4 = 32768, 4096               # cfg4
N5 = 1 << 30                       # cfg5
ADAMW = (1e-3, 0.9, 0.999, 1e-8, 0.01, 10)
BYTES = {
    "add_mul_scalar": 12 * N1,
    "sum": 4 * N2,
    "softmax": 8 * R4 * C4,
    "adamw": 28 * N5,
}
OPS = list(BYTES)
FALLBACK_HBM_GBS = 6650.0


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
    """nvidia-smi samples of this GPU's clocks during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = Path(os.environ.get("TMPDIR", "/tmp")) / f"rt_clocks_{os.getpid()}.csv"

    def __enter__(self):
        try:
            self.f = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-i", str(self.gpu), "-lms", "200"], stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
            self.f.close()

    def summary(self) -> dict:
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
                "samples": len(rows)}


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
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--ops", default=",".join(OPS),
                    help="subset of ops in the step (profiling); the JSON line needs all four")
    ap.add_argument("--small", action="store_true",
                    help="profiling case: sum 2^26, softmax 8192x4096, adamw 4x2^26 (all > L2)")
    args = ap.parse_args()
    if args.small:
        global N2, R4, N5
        N2, R4, N5 = 1 << 26, 8192, 1 << 26
        BYTES.update(sum=4 * N2, softmax=8 * R4 * C4, adamw=28 * N5)
        args.no_e2e = args.no_cpu_baseline = True
    if args.impl == "reference":
        run_reference(args)
        return
    args.warmup = max(args.warmup, 3)

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

    sum_out = c_double()
    sharded = None
    if world > 1 and "sum" in ops:
        from rusttorch_b200 import sharded as sh
        sharded = sh.ShardedReducer(lib, rank, world)

    def run_op(op):
        if op == "add_mul_scalar":
            N.check(lib.rtc_add_mul_scalar(D["a"].ref, D["b"].ref, 0.5, D["c"].ref))
        elif op == "sum":
            if sharded is None:
                N.check(lib.rtc_sum(D["x2"].ref, byref(sum_out)))
            else:
                sum_out.value = sharded.sum(D["x2"])
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
                  "frac_of_measured_peak": BYTES[o] / (op_ms[o] * 1e-3) / 1e9 / peak}
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
    if sharded is not None:
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
    if sharded is not None:
        sharded.close()
    if world > 1:
        dist.destroy_process_group()


def run_e2e(args, lib, N, torch, D, bufs, rank, world, stream):
    """Each step: copy every op's inputs from pinned host memory, run the op
    through the C ABI, copy its result back (c, the sum, y, and p/m/v)."""
    k_e2e = max(1, min(args.steps, 3))
    host = {}
    for k in ("a", "b", "x2", "x4", "p", "g", "m", "v"):
        host[k] = torch.empty(bufs[k].numel(), dtype=torch.float32, pin_memory=True)
        host[k].copy_(bufs[k])
    out = {k: torch.empty(bufs[k].numel(), dtype=torch.float32, pin_memory=True)
           for k in ("c", "y4")}
    h2d = sum(host[k].numel() * 4 for k in host)
    d2h = (out["c"].numel() + out["y4"].numel() + 3 * N5) * 4 + 8
    sum_out = c_double()
    lr, b1, b2, eps, wd, t = ADAMW

    def step():
        bufs["a"].copy_(host["a"], non_blocking=True)
        bufs["b"].copy_(host["b"], non_blocking=True)
        N.check(lib.rtc_add_mul_scalar(D["a"].ref, D["b"].ref, 0.5, D["c"].ref))
        out["c"].copy_(bufs["c"], non_blocking=True)
        bufs["x2"].copy_(host["x2"], non_blocking=True)
        N.check(lib.rtc_sum(D["x2"].ref, byref(sum_out)))
        bufs["x4"].copy_(host["x4"], non_blocking=True)
        N.check(lib.rtc_softmax(D["x4"].ref, 1, D["y4"].ref))
        out["y4"].copy_(bufs["y4"], non_blocking=True)
        for k in "pgmv":
            bufs[k].copy_(host[k], non_blocking=True)
        N.check(lib.rtc_adamw_update(D["p"].ref, D["g"].ref, D["m"].ref, D["v"].ref, lr, b1, b2,
                                     eps, wd, t, D["p"].ref, D["m"].ref, D["v"].ref))
        for k in "pmv":
            host[k].copy_(bufs[k], non_blocking=True)

    step()
    torch.cuda.synchronize()
    import torch.distributed as dist
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(k_e2e):
        step()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / k_e2e
    if world > 1:
        tt = torch.tensor([ms], dtype=torch.float64, device="cuda")
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms = float(tt[0])
    value = sum(BYTES.values()) * world / (ms * 1e-3) / 1e9
    return {"value": value, "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "ms_per_step": ms, "steps": k_e2e,
            "path": "pinned host buffers -> cudaMemcpyAsync -> C-ABI op -> cudaMemcpyAsync back"}


if __name__ == "__main__":
    main()
