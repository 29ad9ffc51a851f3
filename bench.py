#!/usr/bin/env python3
"""Benchmark of the CHPE quantized dequant-matmul hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload NAME]

Prints ONE JSON line (rank 0).  Workloads (synthetic, seeded; no dataset):
  q8_gemv   y[1,12288] = x[1,4096] . dequant(W)^T, W int8 with an fp16 scale per
            32 along K (scales 0.02/127*exp(N(0,0.25))), x fp32 N(0,1), y fp32.
            metric: algorithmic HBM GB/s of the GEMV.
A "step" is one GEMV call (activation-fragment prep + GEMV kernel); the K timed
steps run as one CUDA graph.  Inputs are resident in HBM for `value`; `e2e`
runs the same step eagerly through the public
API with pinned host buffers (host->device x, device->host y inside the timed
region).  Weights rotate over enough copies (> 2x the 126 MB L2) that every
step streams its weights from HBM.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

L2_BYTES = 126 * 1024 * 1024


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained"), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 20 ms across the measurement window."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "20"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = max(mx, float(f[2]))
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


# ----------------------------------------------------------------------------
# workloads
# ----------------------------------------------------------------------------

def q8_gemv_inputs(rng, N=12288, K=4096):
    codes = rng.integers(-127, 128, (N, K), dtype=np.int8)
    scales = (0.02 / 127 * np.exp(rng.normal(0, 0.25, (N, K // 32)))).astype(np.float16)
    x = rng.standard_normal((1, K)).astype(np.float32)
    return codes, scales, x


def q8_gemv_bytes(N=12288, K=4096, M=1):
    return N * K + N * (K // 32) * 2 + M * K * 4 + M * N * 4


def run_ours(args, rank, world, local_rank):
    import torch
    from chpe_qwen35_hybrid_engine_b200 import SCHEME_I8_GROUP_F16, Context

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    ctx = Context(local_rank)
    rng = np.random.default_rng(0)
    N, K, M = 12288, 4096, 1
    codes, scales, x = q8_gemv_inputs(rng, N, K)
    algo = q8_gemv_bytes(N, K, M)
    n_copies = args.copies or max(2, int(np.ceil(3 * L2_BYTES / (N * K))))
    tens = [ctx.upload_matrix(8, SCHEME_I8_GROUP_F16, codes, scales, rows=N, cols=K, group=32)
            for _ in range(n_copies)]
    xd = torch.from_numpy(x).to(dev)
    yd = torch.empty((M, N), dtype=torch.float32, device=dev)
    st = torch.cuda.current_stream(dev)

    def step(i):
        ctx.gemv(tens[i % n_copies], xd, out=yd, stream=st)

    for i in range(args.warmup):
        step(i)
    torch.cuda.synchronize()
    dist_barrier(world)

    clk = ClockSampler(local_rank).__enter__()
    time.sleep(0.1)
    # device-timed region: the K steps run as one CUDA graph (a decode step is
    # replayed as a graph); bracketed by barrier + synchronize
    graph = torch.cuda.CUDAGraph()
    gst = torch.cuda.Stream(dev)
    gst.wait_stream(st)
    with torch.cuda.graph(graph, stream=gst):
        for i in range(args.steps):
            ctx.gemv(tens[i % n_copies], xd, out=yd, stream=gst)
    graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    dist_barrier(world)
    torch.cuda.synchronize()
    rst = torch.cuda.current_stream(dev)  # CUDAGraph.replay() launches on the current stream
    e0.record(rst)
    graph.replay()
    e1.record(rst)
    torch.cuda.synchronize()
    dist_barrier(world)
    ms_total = e0.elapsed_time(e1)
    ms_total = dist_max(ms_total, world)
    ms_step = ms_total / args.steps
    del graph

    # dominant-kernel duration: events bracketing only the GEMV kernel launch
    kern_ms = kernel_times_q8(ctx, tens, xd, yd, st, args.steps, n_copies)

    # end to end through the public API with pinned host buffers
    xh = torch.from_numpy(x).pin_memory()
    yh = torch.empty((M, N), dtype=torch.float32).pin_memory()
    xd2 = torch.empty_like(xd)
    for i in range(args.warmup):
        xd2.copy_(xh, non_blocking=True)
        ctx.gemv(tens[i % n_copies], xd2, out=yd, stream=st)
        yh.copy_(yd, non_blocking=True)
    torch.cuda.synchronize()
    dist_barrier(world)
    e2, e3 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e2.record(st)
    for i in range(args.steps):
        xd2.copy_(xh, non_blocking=True)
        ctx.gemv(tens[i % n_copies], xd2, out=yd, stream=st)
        yh.copy_(yd, non_blocking=True)
    e3.record(st)
    torch.cuda.synchronize()
    e2e_ms = dist_max(e2.elapsed_time(e3), world) / args.steps
    clk.__exit__()

    peaks = measured_peaks()
    kern_avg = statistics.mean(kern_ms)
    achieved = algo / (kern_avg * 1e-3) / 1e9
    value = world * algo / (ms_step * 1e-3) / 1e9
    line = {
        "metric": "quantized GEMV HBM GB/s (Q8 int8 g32 fp16-scale, config 0)",
        "value": round(value, 2),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_step, 6),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "int8 codes x fp32 activations (fp16 tensor-core operands, fp32 accumulate)",
        "data": "synthetic (seeded: int8 U[-127,127], fp16 scales 0.02/127*exp(N(0,0.25)), x N(0,1))",
        "config": {"workload": "q8_gemv", "N": N, "K": K, "M": M, "group": 32,
                   "l2": f"weights rotate over {n_copies} copies ({n_copies * N * K / 2**20:.0f} MiB > 2x L2)",
                   "parallelism": "replicas" if world > 1 else "single"},
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": round(achieved / peaks["hbm_gbs"], 4), "traffic": None,
                     "peak_source": peaks["source"], "kernel": "gemv_kernel", "kernel_us": round(kern_avg * 1e3, 3),
                     "algorithmic_bytes": algo},
        "e2e": {"value": round(world * algo / (e2e_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
                "h2d_bytes_per_step": int(M * K * 4), "d2h_bytes_per_step": int(M * N * 4)},
        "gpu_launches": 2 * args.steps,
        "clocks": clk.summary(),
    }
    if rank == 0 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline_q8(codes, scales, x, algo)
    ctx.close()
    return line


def kernel_times_q8(ctx, tens, xd, yd, st, steps, n_copies):
    """Duration of the GEMV kernel alone: the activation fragments are prepared
    once (chpe_xfrag_*), then `steps` GEMV launches run as one CUDA graph on a
    stream of their own, timed with CUDA events on that stream."""
    import torch
    from chpe_qwen35_hybrid_engine_b200 import X_F32
    gst = torch.cuda.Stream()
    gst.wait_stream(st)
    xf = ctx.xfrag(tens[0], xd.shape[0], X_F32)
    ctx.xfrag_fill(xf, xd, stream=gst)
    for i in range(3):
        ctx.gemv_xfrag(tens[i % n_copies], xf, yd, stream=gst)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=gst):
        for i in range(steps):
            ctx.gemv_xfrag(tens[i % n_copies], xf, yd, stream=gst)
    graph.replay()
    torch.cuda.synchronize()
    times = []
    rst = torch.cuda.current_stream()  # CUDAGraph.replay() launches on the current stream
    for _ in range(3):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(rst)
        graph.replay()
        b.record(rst)
        torch.cuda.synchronize()
        times.append(a.elapsed_time(b) / steps)
    del graph
    xf.free()
    return times


def cpu_baseline_q8(codes, scales, x, algo, budget_s=10.0):
    from oracle import oracle as O
    threads = os.cpu_count() or 1
    t0 = time.perf_counter()
    n = 0
    while True:
        O.gemv_grouped(codes, scales, None, 32, x, num_workers=threads)
        n += 1
        if time.perf_counter() - t0 > budget_s:
            break
    dt = (time.perf_counter() - t0) / n
    return {"value": round(algo / dt / 1e9, 3), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"{n} full config-0 GEMVs (12288x4096) by the C oracle, fp64 accumulation, {threads} threads"}


def run_reference(args, rank, world):
    """CPU reference arm: the oracle port of the reference path on the host cores."""
    if rank != 0:
        return None
    rng = np.random.default_rng(0)
    codes, scales, x = q8_gemv_inputs(rng)
    algo = q8_gemv_bytes()
    from oracle import oracle as O
    threads = os.cpu_count() or 1
    for _ in range(args.warmup):
        O.gemv_grouped(codes, scales, None, 32, x, num_workers=threads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        O.gemv_grouped(codes, scales, None, 32, x, num_workers=threads)
    dt = (time.perf_counter() - t0) / args.steps
    v = round(algo / dt / 1e9, 3)
    return {
        "impl": "reference",
        "metric": "quantized GEMV HBM GB/s (Q8 int8 g32 fp16-scale, config 0)",
        "value": v, "unit": "GB/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(dt * 1e3, 4), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "int8 codes x fp32 activations (fp64 accumulate)", "data": "synthetic (seeded)",
        "config": {"workload": "q8_gemv", "N": 12288, "K": 4096, "M": 1, "group": 32},
        "cpu_baseline": {"value": v, "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": "full config-0 GEMV per step (C restatement; the Zig reference needs a Zig 0.17-dev toolchain absent here)"},
        "e2e": {"value": v, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


# ----------------------------------------------------------------------------
# distributed plumbing
# ----------------------------------------------------------------------------

def dist_barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def dist_max(v, world):
    if world <= 1:
        return v
    import torch
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="q8_gemv")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--copies", type=int, default=0, help="weight copies to rotate (default: > 3x L2)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        line = run_reference(args, rank, world)
        if line is not None:
            print(json.dumps(line), flush=True)
        return 0

    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    line = run_ours(args, rank, world, local_rank)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
