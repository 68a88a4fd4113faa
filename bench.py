#!/usr/bin/env python
"""Benchmark of the quantized decode GEMV hot path.

One step = one batch-1 GEMV sweep over the five Phi-4-mini projection shapes
(Q4_K weights, K->N: qkv 3072->5120, o 3072->3072, gate_up 3072->16384,
down 8192->3072, lm_head 3072->200064), seeds 0-4, x ~ N(0,1). Metric:
algorithmic bytes (GGUF weight bytes + 4K input + 4N output) per second.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Multi-GPU (torchrun, one rank per GPU): every weight is row-sharded over the
ranks (contiguous row slices); each rank runs its GEMV slice and the output
vectors are all-gathered, so total work is fixed ("strong" scaling).

--impl reference times the reference CpuVm mat-vec algorithm (the C
restatement in oracle/, all host threads) on the same workload.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

SHAPES = [("qkv", 5120, 3072, 0), ("o", 3072, 3072, 1), ("gate_up", 16384, 3072, 2), ("down", 3072, 8192, 3),
          ("lm_head", 200064, 3072, 4)]
WTYPE = 12  # Q4_K
METRIC = "quant GEMV weight GB/s (Q4_K batch-1 sweep, Phi-4-mini shapes)"
FALLBACK_HBM_GBS = 6650.0


def q4k_bytes(rows: int, cols: int) -> int:
    return rows * cols // 256 * 144


def step_bytes(shapes) -> int:
    return sum(q4k_bytes(n, k) + 4 * k + 4 * n for _, n, k, _ in shapes)


def measured_peak() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs)"
        except Exception:
            pass
    return FALLBACK_HBM_GBS, "fallback 6.65 TB/s"


def committed_traffic() -> dict | None:
    p = ROOT / "profiles" / "gemv_q4_k_sweep_traffic.json"
    if p.exists():
        try:
            return json.loads(p.read_text())
        except Exception:
            return None
    return None


class ClockSampler:
    """Samples nvidia-smi clocks / throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc:
            self.proc.terminate()
            try:
                self.out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()
                self.out = ""
        return False

    def summary(self) -> dict:
        out = getattr(self, "out", "") or ""
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    return world, rank, local


def cpu_reference_sweep(shapes, weights, xs, threads: int) -> float:
    import oracle
    t0 = time.perf_counter()
    for (name, n, k, _), blob, x in zip(shapes, weights, xs):
        oracle.matvec(WTYPE, blob, x, n, k, threads)
    return time.perf_counter() - t0


def make_inputs(shapes):
    from sharpinference_b200 import native
    weights = [native.synth_weights(WTYPE, seed, n, k, 0.02) for _, n, k, seed in shapes]
    xs = [native.synth_normal(1000 + seed, k, 1.0) for _, n, k, seed in shapes]
    return weights, xs


def run_reference(args) -> None:
    world, rank, _ = dist_env()
    if rank != 0:
        return
    import oracle
    weights, xs = make_inputs(SHAPES)
    threads = oracle.online_cores()
    for _ in range(args.warmup):
        cpu_reference_sweep(SHAPES, weights, xs, threads)
    times = [cpu_reference_sweep(SHAPES, weights, xs, threads) for _ in range(args.steps)]
    total = sum(times)
    value = step_bytes(SHAPES) * args.steps / total / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(1e3 * total / args.steps, 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded N(0,0.02) Q4_K weights, N(0,1) x)",
        "config": {"workload": "config2 Q4_K batch-1 GEMV sweep (Phi-4-mini qkv/o/gate_up/down/lm_head)",
                   "shapes_nk": [[n, k] for _, n, k, _ in SHAPES], "bytes_per_step": step_bytes(SHAPES)},
        "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": f"full sweep x {args.steps} steps; C restatement of CpuHalfMatrixOperators.MatVec "
                                   "(per-row dequantise + FP32 dot, rows parallel)"},
        "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_ours(args) -> None:
    import numpy as np
    import torch
    import torch.distributed as dist
    from sharpinference_b200 import native

    world, rank, local = dist_env()
    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", device_id=torch.device("cuda", local),
                               timeout=__import__("datetime").timedelta(seconds=120))
    ctx = native.Context(local)
    stream = torch.cuda.ExternalStream(ctx.stream, device=torch.device("cuda", local))

    # Row shard of every shape for this rank (contiguous slices).
    shards = []
    for name, n, k, seed in SHAPES:
        r0 = n * rank // world
        r1 = n * (rank + 1) // world
        shards.append((name, n, k, seed, r0, r1))
    full = native.synth_weights  # generate the full matrix and keep this rank's rows
    W, X, Y, YS = [], [], [], []
    host_x = []
    for name, n, k, seed, r0, r1 in shards:
        rb = native.row_bytes(WTYPE, k)
        blob = full(WTYPE, seed, n, k, 0.02)
        part = blob[r0 * rb:r1 * rb]
        wb = ctx.buffer(part.nbytes)
        wb.upload(part)
        x = native.synth_normal(1000 + seed, k, 1.0)
        xb = ctx.buffer(x.nbytes)
        xb.upload(x)
        yb = ctx.buffer((r1 - r0) * 4)
        W.append(wb), X.append(xb), Y.append(yb), host_x.append(x)
        YS.append(torch.empty(n, dtype=torch.float32, device=f"cuda:{local}") if world > 1 else None)
        del blob

    def step(events=None):
        with torch.cuda.stream(stream):
            for i, (name, n, k, seed, r0, r1) in enumerate(shards):
                if events is not None:
                    events[i][0].record(stream)
                ctx.matvec(WTYPE, W[i], X[i], Y[i], r1 - r0, k)
                if events is not None:
                    events[i][1].record(stream)

    if world > 1:
        raise SystemExit("multi-GPU bench path is not built yet")

    for _ in range(max(args.warmup, 3)):
        step()
    ctx.synchronize()
    torch.cuda.synchronize()

    per_launch = [[(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
                   for _ in shards] for _ in range(args.steps)]
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    sampler = ClockSampler(local)
    with sampler:
        time.sleep(0.25)
        start.record(stream)
        for s in range(args.steps):
            step(per_launch[s])
        stop.record(stream)
        stop.synchronize()
    torch.cuda.synchronize()
    total_ms = start.elapsed_time(stop)
    launch_ms = [[a.elapsed_time(b) for a, b in per_launch[s]] for s in range(args.steps)]
    bytes_step = step_bytes(SHAPES)
    value = bytes_step * args.steps / (total_ms * 1e-3) / 1e9

    # dominant kernel: the staged Q4_K GEMV (all five launches of a step)
    kern_ms = sum(sum(l) for l in launch_ms) / (args.steps * len(shards))
    kern_bytes = bytes_step / len(shards)
    achieved = kern_bytes / (kern_ms * 1e-3) / 1e9
    peak, peak_src = measured_peak()
    per_shape = {}
    for i, (name, n, k, seed, r0, r1) in enumerate(shards):
        ms = statistics.median(launch_ms[s][i] for s in range(args.steps))
        b = q4k_bytes(n, k) + 4 * k + 4 * n
        per_shape[name] = {"us": round(ms * 1e3, 2), "GB/s": round(b / (ms * 1e-3) / 1e9, 1),
                           "frac": round(b / (ms * 1e-3) / 1e9 / peak, 3)}
    traffic = committed_traffic()

    # e2e: the public C-ABI call with host buffers; x uploaded from pinned
    # memory and y read back to pinned memory inside the timed region.
    import ctypes as C
    pinned_x, pinned_y = [], []
    for i, (name, n, k, seed, r0, r1) in enumerate(shards):
        px, py = C.c_void_p(), C.c_void_p()
        native.call("si_host_alloc_pinned", k * 4, C.byref(px))
        native.call("si_host_alloc_pinned", (r1 - r0) * 4, C.byref(py))
        C.memmove(px, host_x[i].ctypes.data, k * 4)
        pinned_x.append(px), pinned_y.append(py)

    def e2e_step():
        for i, (name, n, k, seed, r0, r1) in enumerate(shards):
            native.call("si_buffer_upload_async", ctx.handle, X[i].handle, 0, pinned_x[i], k * 4)
            ctx.matvec(WTYPE, W[i], X[i], Y[i], r1 - r0, k)
            native.call("si_buffer_readback_async", ctx.handle, Y[i].handle, 0, pinned_y[i], (r1 - r0) * 4)
        ctx.synchronize()

    for _ in range(max(args.warmup, 3)):
        e2e_step()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    e0.record(stream)
    for _ in range(args.steps):
        e2e_step()
    e1.record(stream)
    e1.synchronize()
    wall = time.perf_counter() - t0
    e2e_ms = max(e0.elapsed_time(e1), wall * 1e3)
    e2e_value = bytes_step * args.steps / (e2e_ms * 1e-3) / 1e9
    h2d = sum(4 * k for _, n, k, _ in SHAPES)
    d2h = sum(4 * n for _, n, k, _ in SHAPES)
    # sanity: last e2e result equals the device-resident result
    y_dev = np.frombuffer(Y[-1].readback(), dtype=np.float32)
    y_host = np.ctypeslib.as_array(C.cast(pinned_y[-1], C.POINTER(C.c_float)), shape=(shards[-1][5] - shards[-1][4],))
    assert np.array_equal(y_dev, y_host)
    for p in pinned_x + pinned_y:
        native.call("si_host_free_pinned", p)

    cpu = None
    if rank == 0 and not args.no_cpu_baseline:
        import oracle
        weights, xs = make_inputs(SHAPES)
        threads = oracle.online_cores()
        cpu_reference_sweep(SHAPES, weights, xs, threads)  # warm
        t_budget, reps, spent = 10.0, 0, 0.0
        while spent < t_budget and reps < 50:
            spent += cpu_reference_sweep(SHAPES, weights, xs, threads)
            reps += 1
        cpu = {"value": round(bytes_step * reps / spent / 1e9, 3), "unit": "GB/s", "cores": threads, "kind": "port",
               "sample": f"{reps} full sweeps ({spent:.1f} s); C restatement of CpuHalfMatrixOperators.MatVec "
                         "(per-row dequantise + FP32 dot, rows parallel over all host threads)"}

    err = native.device_error_take(local)
    if err:
        raise SystemExit(f"device error word {err:#x}")
    clocks = sampler.summary()
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(total_ms / args.steps, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded N(0,0.02) weights quantized to Q4_K; x ~ N(0,1))",
            "config": {"workload": "config2 Q4_K batch-1 GEMV sweep (Phi-4-mini qkv/o/gate_up/down/lm_head)",
                       "shapes_nk": [[n, k] for _, n, k, _ in SHAPES], "bytes_per_step": bytes_step,
                       "l2": "inputs larger than L2 (402 MB of weights streamed per step)",
                       "parallelism": f"row-shard x{world}" if world > 1 else "single GPU"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_source": peak_src,
                         "kernel": "gemv_staged_kernel<Q4_K>",
                         "traffic": traffic.get("bytes_per_launch") if traffic else None,
                         "per_shape": per_shape},
            "cpu_baseline": cpu,
            "e2e": {"value": round(e2e_value, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h},
            "gpu_launches": len(shards) * args.steps,
            "clocks": clocks,
        }
        print(json.dumps(line), flush=True)
    ctx.close()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
