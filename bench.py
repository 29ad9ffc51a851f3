#!/usr/bin/env python3
"""Benchmark of the CHPE quantized dequant-matmul hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload NAME]

Prints ONE JSON line (rank 0).  Workloads (synthetic and seeded; there is no
dataset and no checkpoint):

  decode_72b (default)  Qwen2.5-72B-shaped decode (80 GQA layers, hidden 8192,
                        FFN 29568, vocab 152064), 4-bit weights with an fp16
                        scale and zero per 64 columns, tensor parallel over the
                        N GPUs (the library's one-shot NVLink all-reduce kernel
                        after o and down), batch 1, over a 1024-token seeded
                        context prefilled through the engine (GQA attention
                        with RoPE over an fp32 KV cache); the batch-8 verify
                        step is reported beside it.  metric: tokens/s for the
                        whole job.  At N = 1 the line also carries the
                        Qwen3.5-9B-shaped decode (8-bit, fp16 scale per 32;
                        Gated-DeltaNet recurrence and gated GQA attention, 512
                        context tokens) at batch 1 and the batch-4 / batch-8
                        verify steps, the single Q8 GEMV (q8_gemv), the 4-bit /
                        2-bit GEMV sweep and the prefill GEMMs.
  decode_9b             the Qwen3.5-9B-shaped decode alone (N > 1: replicas).
  gemv                  one quantized GEMV y[M,N] = x[M,K] . dequant(W)^T
                        (--bits 8|4|2 --rows N --cols K --batch M --x f32|bf16);
                        metric: algorithmic HBM GB/s.  `q8_gemv` is the
                        12288x4096 int8 GEMV (fp16 scale per 32) at batch 1.
  prefill               the prefill dequant-GEMM (tcgen05), metric TFLOP/s.

A decode step is one token per row: embedding, every layer, final norm, LM
head and argmax; with M rows the rows are consecutive positions (speculative
verification).  Timed steps replay one CUDA graph per step and feed each
step's argmax into the next on the device; the weights (7 GB for the 9B shape,
40 GB / N for the 72B shape) are far larger than the 126 MB L2, so every step
streams them from HBM.  `e2e` runs the same steps with the token copied in from
pinned host memory and the argmax copied back to the host every step.  The
roofline is that of the GEMV kernel: every GEMV of one step is captured on its
own (activation fragments prepared beforehand) and its algorithmic bytes
(packed codes + scales/zeros + activations read + outputs written) are divided
by the replayed GEMV time.  The CPU baseline is the reference engine's CPU
step restated in C (oracle/cpu_baseline.c), whole steps on the host's cores.
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

# DRAM traffic (dram__bytes_read.sum + dram__bytes_write.sum) of the dominant
# kernel, per launch, from single-launch ncu captures summarised under
# profiles/.  A decode step is too large to capture whole: its traffic is the
# step's algorithmic GEMV bytes times the traffic / algorithmic ratio of the
# captured GEMV of the same format (Q4 g64 29568 x 8192, Q8 g32 12288 x 4096,
# batch 1).
NCU_TRAFFIC = {
    ("gemv", 8, 12288, 4096, 1, "f32"): 53_648_128,
    ("gemv", 4, 29568, 8192, 1, "f32"): 142_191_104,
    ("gemv", 4, 29568, 8192, 8, "f32"): 142_469_120,
    ("prefill", 8, 12288, 4096, 2048): 138_023_168,
}
Q4_TRAFFIC_RATIO = 142_191_104 / 136_400_384
Q8_TRAFFIC_RATIO = 53_648_128 / 53_542_912
DECODE_METRIC = "decode tokens/s (quantized GEMV path; GEMV HBM GB/s vs peak in roofline)"


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

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "20"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            threading.Thread(target=self._read, daemon=True).start()
        except (OSError, FileNotFoundError):
            self.proc = None
        time.sleep(0.1)
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
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


def timed_replays(replay, steps, world, dev):
    """`steps` calls of replay(), bracketed by barrier + synchronize on both
    sides; device time (ms) from CUDA events on the current stream (where
    CUDAGraph.replay() launches), max over ranks."""
    import torch
    rst = torch.cuda.current_stream(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize(dev)
    dist_barrier(world)
    torch.cuda.synchronize(dev)
    e0.record(rst)
    for _ in range(steps):
        replay()
    e1.record(rst)
    torch.cuda.synchronize(dev)
    dist_barrier(world)
    return dist_max(e0.elapsed_time(e1), world)


# ----------------------------------------------------------------------------
# decode workloads
# ----------------------------------------------------------------------------

def gemv_step_profile(ctx, eng, M, reps, dev):
    """Every GEMV of one step as the engine issues it at this row count
    (activation fragments prepared beforehand, one fragment set per input),
    captured as one graph and replayed `reps` times.  Returns (GEMV ms per
    step, algorithmic bytes per step, GEMV launches per step)."""
    import torch
    from chpe_qwen35_hybrid_engine_b200 import X_F32
    groups = []  # (tensors, mode)
    for lw in eng.layers:
        p = lw.proj
        groups.append(([p["q"], p["k"], p["v"]] if "q" in p else [p["qkv"], p["z"]], 0))
        groups.append(([p["o"] if "q" in p else p["out"]], 0))
        groups.append(([p["gate"], p["up"]], 1 if M == 1 else 0))
        groups.append(([p["down"]], 0))
    groups.append(([eng.head], 0))
    rows = max(t.rows for ts, _ in groups for t in ts)
    ys = [torch.empty(M, rows, device=dev) for _ in range(3)]
    xfs = {}
    for ts, _ in groups:
        key = (ts[0].cols, ts[0].bits)
        if key not in xfs:
            xf = ctx.xfrag(ts[0], M, X_F32)
            ctx.xfrag_fill(xf, torch.randn(M, ts[0].cols, device=dev))
            xfs[key] = xf
    torch.cuda.synchronize(dev)
    st = torch.cuda.Stream(dev)
    st.wait_stream(torch.cuda.current_stream(dev))

    def issue():
        for ts, mode in groups:
            xf = xfs[(ts[0].cols, ts[0].bits)]
            if mode == 1:
                ctx.gemv_gateup_swiglu_xfrag(ts[0], ts[1], xf, ys[0], stream=st)
            elif len(ts) > 1:
                ctx.gemv_multi_xfrag(ts, xf, ys[:len(ts)], stream=st)
            else:
                ctx.gemv_xfrag(ts[0], xf, ys[0], stream=st)

    with torch.cuda.stream(st):
        issue()
    torch.cuda.synchronize(dev)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=st):
        issue()
    for _ in range(3):
        graph.replay()
    ms = timed_replays(graph.replay, reps, 1, dev) / reps
    del graph
    for xf in xfs.values():
        xf.free()
    nbytes = 0
    for ts, mode in groups:
        nbytes += sum(t.device_bytes + M * t.rows * 4 for t in ts) + M * ts[0].cols * 4
        if mode == 1:
            nbytes -= M * ts[1].rows * 4  # one output for gate and up
    return ms, nbytes, len(groups)


def exchange_step_profile(tp, M, reps, world, dev):
    """The tensor-parallel exchanges of one step alone -- the all-reduce after
    O and after down of every layer and the LM head's argmax merge -- on the
    step's comm object, captured as one graph and replayed `reps` times
    (every rank replays the same sequence).  Returns ms per step, max over
    ranks."""
    import torch
    H = tp.geom.hidden
    part = torch.randn(M, H, device=dev)
    hidden = torch.zeros(M, H, device=dev)
    idx = torch.zeros(M, dtype=torch.int32, device=dev)
    val = torch.zeros(M, device=dev)
    st = torch.cuda.Stream(dev)
    st.wait_stream(torch.cuda.current_stream(dev))

    def issue():
        for _ in range(2 * tp.geom.n_layers):
            tp.comm.allreduce_residual(part, hidden, M * H, stream=st)
        tp.comm.argmax_merge(idx, val, M, tp.v0, stream=st)

    with torch.cuda.stream(st):
        issue()
    torch.cuda.synchronize(dev)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=st):
        issue()
    for _ in range(3):
        graph.replay()
    ms = timed_replays(graph.replay, reps, world, dev) / reps
    del graph
    return ms


def decode_line(eng, stepper, M, args, world, dev, label, context_len, profile=True):
    """Graph-replayed greedy decode at M rows after a seeded context of
    context_len uniform token ids has been prefilled through the engine (8
    positions per step); returns a dict of figures."""
    import torch
    from chpe_qwen35_hybrid_engine_b200 import kernel_launches
    b = eng.buf
    rng = np.random.default_rng(0)
    context = rng.integers(0, eng.geom.vocab, context_len).astype(np.int32)  # seeded uniform token ids
    first = np.array([(int(context[-1]) + 7 * i) % eng.geom.vocab for i in range(M)], np.int32)
    stepper.reset()
    t0 = time.perf_counter()
    stepper.prefill(context, M=8)
    prefill_s = time.perf_counter() - t0
    pos0 = int(eng.pos.item())
    b["tokens"][:M].copy_(torch.from_numpy(first).to(dev))
    snap = eng._snapshot()
    n0 = kernel_launches()
    torch.cuda.nvtx.range_push(f"{label}_step")  # one eager step: the range a launch-list capture selects
    stepper.step(M)
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize(dev)
    launches_per_step = kernel_launches() - n0
    eng._restore(snap)
    b["tokens"][:M].copy_(torch.from_numpy(first).to(dev))
    graph = stepper.capture(M)
    st = torch.cuda.Stream(dev)
    st.wait_stream(torch.cuda.current_stream(dev))
    feed = torch.cuda.CUDAGraph()  # next step's tokens = this step's argmax, on the device
    with torch.cuda.graph(feed, stream=st):
        b["tokens"][:M].copy_(b["argmax"][:M])

    def replay():
        graph.replay()
        feed.replay()

    for _ in range(args.warmup):
        replay()
    ms_step = timed_replays(replay, args.steps, world, dev) / args.steps
    # end to end: the step's token comes from pinned host memory and its argmax goes back
    tok_h = torch.from_numpy(first.copy()).pin_memory()
    out_h = torch.zeros(M, dtype=torch.int32).pin_memory()
    rst = torch.cuda.current_stream(dev)

    def e2e_step():
        b["tokens"][:M].copy_(tok_h, non_blocking=True)
        graph.replay()
        out_h.copy_(b["argmax"][:M], non_blocking=True)
        rst.synchronize()
        tok_h.copy_(out_h)

    for _ in range(args.warmup):
        e2e_step()
    e2e_ms = timed_replays(e2e_step, args.steps, world, dev) / args.steps
    del feed
    stepper.graphs.clear()
    del graph
    pos1 = int(eng.pos.item())
    out = {"label": label, "rows": M, "tok_s": round(M / (ms_step * 1e-3), 2),
           "ms_per_step": round(ms_step, 4), "e2e_tok_s": round(M / (e2e_ms * 1e-3), 2),
           "e2e_ms_per_step": round(e2e_ms, 4), "kernel_launches_per_step": int(launches_per_step),
           "weight_bytes": int(eng.n_weight_bytes()), "context_tokens": int(context_len),
           "positions": [pos0, pos1], "context_prefill_s": round(prefill_s, 3)}
    if profile:
        gms, gbytes, glaunch = gemv_step_profile(eng.ctx, eng, M, max(5, min(args.steps, 20)), dev)
        gms = dist_max(gms, world)
        out.update({"gemv_ms_per_step": round(gms, 4), "gemv_bytes_per_step": int(gbytes),
                    "gemv_launches_per_step": glaunch, "gemv_gbs": round(gbytes / (gms * 1e-3) / 1e9, 1)})
        # where the step's time goes: the GEMVs timed alone, and the rest of
        # the step (fills -- with tensor parallelism the ones that carry the
        # exchanges --, mixers, norms, argmax, launch gaps); beside it the
        # step's exchanges run alone as separate all-reduce kernels, the form
        # the step itself does not use
        bd = {"gemv_ms": round(gms, 4), "other_ms": round(ms_step - gms, 4)}
        if getattr(stepper, "comm", None) is not None:
            bd["exchange_kernels_alone_ms"] = round(
                exchange_step_profile(stepper, M, max(5, min(args.steps, 20)), world, dev), 4)
        out["breakdown"] = bd
    return out


def _decode_geometry(which, args):
    """The benchmark model with the real token mixers and a KV cache sized for
    the context plus every step the measurement runs (8 rows at most)."""
    import dataclasses
    from chpe_qwen35_hybrid_engine_b200.engine import QWEN25_72B, QWEN35_9B
    base, ctx_len = (QWEN25_72B, 1024) if which == "decode_72b" else (QWEN35_9B, 512)
    if args.context is not None:
        ctx_len = max(8, args.context)
    need = ctx_len + 8 * (2 * (args.warmup + args.steps) + 8)
    return dataclasses.replace(base, mixer="real", max_seq=(need + 255) // 256 * 256), ctx_len


def decode_config(which, world, ctx_len=None):
    """The `config` of a decode line (both arms)."""
    if ctx_len is None:
        ctx_len = 1024 if which == "decode_72b" else 512
    if which == "decode_72b":
        return {"workload": "decode_72b",
                "model": "Qwen2.5-72B-shaped: 80 GQA layers, hidden 8192, FFN 29568 SwiGLU, 64/8 heads of 128, "
                         "vocab 152064",
                "weights": "4-bit codes, fp16 scale + zero per 64 columns (seeded random codes and scales)",
                "tensor_parallel": world, "global_batch": 1,
                "context": f"{ctx_len} seeded uniform token ids prefilled through the engine (RoPE, fp32 KV cache); "
                           "decode continues from there",
                "parallelism": f"tp{world}", "l2": "40 GB / N of weights per step >> 126 MB L2"}
    return {"workload": "decode_9b",
            "model": "Qwen3.5-9B-shaped hybrid: 24 Gated DeltaNet + 8 gated GQA layers, hidden 4096, FFN 12288, "
                     "vocab 151936",
            "weights": "8-bit codes, fp16 scale per 32 columns (random-init N(0,0.02))",
            "context": f"{ctx_len} seeded uniform token ids prefilled through the engine",
            "global_batch": world, "parallelism": f"replicas{world}", "l2": "7 GB of weights per step >> 126 MB L2"}


def run_decode(args, rank, world, local_rank, which):
    import torch
    from chpe_qwen35_hybrid_engine_b200 import Context
    from chpe_qwen35_hybrid_engine_b200.engine import build_random
    from chpe_qwen35_hybrid_engine_b200.tp import TensorParallelEngine
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    peaks = measured_peaks()
    clk = ClockSampler(local_rank)
    extra = {}
    ctx = Context(local_rank)
    geom, ctx_len = _decode_geometry(which, args)
    if which == "decode_72b":
        tp = TensorParallelEngine(ctx, geom, "q4g64", rank, world, seed=0, max_rows=8, random_codes=True)
        tp.eng.push_exchange = args.exchange == "push"
        clk.start()
        main = decode_line(tp.eng, tp, 1, args, world, dev, f"72b_tp{world}_b1", ctx_len)
        clk.stop()
        extra["decode_72b_b8"] = decode_line(tp.eng, tp, 8, args, world, dev, f"72b_tp{world}_b8", ctx_len)
        tp.graphs.clear()
        if tp.comm is not None:
            tp.comm.close()
        del tp
        config = decode_config(which, world, ctx_len)
        if world > 1:
            config["exchange"] = f"NVLink P2P, tagged words, sent by the {'GEMV' if args.exchange == 'push' else 'fill'}"
        scaling, units = "strong", 1
    else:
        eng, _ = build_random(ctx, geom, "q8g32", seed=rank, max_rows=8)
        clk.start()
        main = decode_line(eng, eng, 1, args, world, dev, "9b_b1", ctx_len)
        clk.stop()
        del eng
        config = decode_config(which, world, ctx_len)
        scaling, units = "weak", world
    ctx.close()
    torch.cuda.empty_cache()
    if which == "decode_72b" and world == 1:
        ctx9 = Context(local_rank)
        g9, c9 = _decode_geometry("decode_9b", args)
        eng9, _ = build_random(ctx9, g9, "q8g32", seed=0, max_rows=8)
        for M in (1, 4, 8):
            extra[f"decode_9b_b{M}"] = decode_line(eng9, eng9, M, args, 1, dev, f"9b_b{M}", c9)
        eng9.graphs.clear()
        del eng9
        ctx9.close()
        torch.cuda.empty_cache()
        if not args.no_sweep:
            extra.update(kernel_sweep(dev, local_rank, peaks))
    achieved = main["gemv_gbs"]
    n_launch = main["kernel_launches_per_step"] * args.steps
    if which == "decode_9b":
        traffic = int(main["gemv_bytes_per_step"] * Q8_TRAFFIC_RATIO)
    else:
        traffic = int(main["gemv_bytes_per_step"] * Q4_TRAFFIC_RATIO)
    line = {
        "metric": DECODE_METRIC, "value": round(main["tok_s"] * units, 2), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": main["ms_per_step"], "higher_is_better": True,
        "scaling": scaling, "vs_baseline": None,
        "dtype": "int4/int8 codes x fp32 activations (fp16 tensor-core operands, fp32 accumulate)",
        "data": "synthetic (seeded random-init weights, seeded uniform token ids)",
        "config": config,
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": round(achieved / peaks["hbm_gbs"], 4), "traffic": traffic,
                     "traffic_unit": "bytes per step (all GEMV launches of one step, per GPU)",
                     "peak_source": peaks["source"],
                     "kernel": "chpe_qgemv_kernel: all GEMVs of one step on one GPU, bytes / GEMV time",
                     "algorithmic_bytes_per_step": main["gemv_bytes_per_step"],
                     "gemv_ms_per_step": main["gemv_ms_per_step"]},
        "e2e": {"value": round(main["e2e_tok_s"] * units, 2), "unit": "tokens/s", "h2d_bytes_per_step": 4,
                "d2h_bytes_per_step": 4},
        "gpu_launches": int(n_launch),
        "clocks": clk.summary(),
        "detail": main,
    }
    line.update(extra)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_decode_baseline(which)
    return line


def kernel_sweep(dev, local_rank, peaks):
    """The single-kernel benchmark configurations at N = 1, each kernel timed
    alone in a CUDA graph over weight copies that rotate through > 3x L2:
    the Q8 GEMV 12288x4096 (q8_gemv), the 4-bit / 2-bit GEMV sweep (K, N) in
    {(4096,4096), (4096,12288), (12288,4096), (4096,151936)} at M = 1/4/8 with
    bf16 activations, and the prefill GEMMs (M = 2048 bf16 tokens; Q8 g32 and
    Q4 g64 weights of (4096,12288), (12288,4096), (4096,6144))."""
    import torch
    from chpe_qwen35_hybrid_engine_b200 import Context
    ctx = Context(local_rank)
    out = {}
    hbm = peaks["hbm_gbs"]
    g = torch.Generator(device=dev)
    g.manual_seed(0)

    def weights(bits, N, K, copies):
        from chpe_qwen35_hybrid_engine_b200 import SCHEME_I8_GROUP_F16, SCHEME_U_GROUP_F16_ZERO
        tens = []
        for _ in range(copies):
            if bits == 8:
                codes = torch.randint(-127, 128, (N, K), dtype=torch.int8, device=dev, generator=g)
                s = (0.02 / 127 * torch.exp(0.25 * torch.randn(N, K // 32, device=dev, generator=g))).half()
                tens.append(ctx.upload_matrix(8, SCHEME_I8_GROUP_F16, codes, s, rows=N, cols=K, group=32))
            else:
                codes = torch.randint(0, 256, (N, K * bits // 8), dtype=torch.uint8, device=dev, generator=g)
                s = (0.02 * 5 / ((1 << bits) - 1) * torch.exp(0.25 * torch.randn(N, K // 64, device=dev,
                                                                                   generator=g))).half()
                mid = (1 << bits) // 2
                z = torch.randint(max(0, mid - 2), mid + 2, (N, K // 64), device=dev, generator=g).half()
                tens.append(ctx.upload_matrix(bits, SCHEME_U_GROUP_F16_ZERO, codes, s, z, rows=N, cols=K, group=64))
        return tens

    def time_graph(issue, reps=3):
        st = torch.cuda.Stream(dev)
        st.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(st):
            issue(st)
        torch.cuda.synchronize(dev)
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr, stream=st):
            issue(st)
        for _ in range(2):
            gr.replay()
        ms = timed_replays(gr.replay, reps, 1, dev) / reps
        del gr
        return ms

    def gemv_case(bits, N, K, M, xdt):
        wb = N * K * bits // 8 + (N * K // 32) * 2 if bits == 8 else N * K * bits // 8 + (N * K // 64) * 4
        copies = max(2, min(64, -(-3 * L2_BYTES // wb)))
        tens = weights(bits, N, K, copies)
        x = torch.randn(M, K, device=dev, generator=g)
        from chpe_qwen35_hybrid_engine_b200 import X_BF16, X_F32
        if xdt == "bf16":
            x = x.to(torch.bfloat16)
        xf = ctx.xfrag(tens[0], M, X_BF16 if xdt == "bf16" else X_F32)
        ctx.xfrag_fill(xf, x)
        y = torch.empty(M, N, device=dev)
        per_graph = max(copies, 8)
        ms = time_graph(lambda st: [ctx.gemv_xfrag(tens[i % copies], xf, y, stream=st) for i in range(per_graph)])
        us = ms * 1e3 / per_graph
        algo = wb + M * K * (2 if xdt == "bf16" else 4) + M * N * 4
        gbs = algo / (us * 1e-6) / 1e9
        xf.free()
        for t in tens:
            t.free()
        torch.cuda.synchronize(dev)
        return {"us": round(us, 3), "gbs": round(gbs, 1), "frac": round(gbs / hbm, 4), "algorithmic_bytes": int(algo),
                "weight_copies": copies}

    out["q8_gemv"] = dict(gemv_case(8, 12288, 4096, 1, "f32"),
                          config="Q8 g32 (fp16 scale per 32), y[1,12288] = x[1,4096] fp32 . W^T")
    sweep = {}
    for bits in (4, 2):
        for K, N in ((4096, 4096), (4096, 12288), (12288, 4096), (4096, 151936)):
            for M in (1, 4, 8):
                sweep[f"q{bits}_k{K}_n{N}_m{M}"] = gemv_case(bits, N, K, M, "bf16")
    out["gemv_sweep"] = {"config": "unsigned 4/2-bit codes, fp16 scale + zero per 64, bf16 x; kernel alone",
                         "peak_gbs": hbm, "cases": sweep}
    pre = {}
    peak_t = peaks["bf16_tflops"]
    for bits in (8, 4):
        for K, N in ((4096, 12288), (12288, 4096), (4096, 6144)):
            wb = N * K * bits // 8
            copies = max(2, min(16, -(-3 * L2_BYTES // wb)))
            tens = weights(bits, N, K, copies)
            M = 2048
            x = torch.randn(M, K, device=dev, generator=g).to(torch.bfloat16)
            y = torch.empty(M, N, device=dev)
            ms = time_graph(lambda st: [ctx.gemm_prefill(tens[i % copies], x, out=y, stream=st)
                                        for i in range(copies)]) / copies
            tf = 2.0 * M * N * K / (ms * 1e-3) / 1e12
            pre[f"q{bits}_k{K}_n{N}"] = {"ms": round(ms, 4), "tflops": round(tf, 1), "frac": round(tf / peak_t, 4)}
            for t in tens:
                t.free()
            torch.cuda.synchronize(dev)
    out["prefill"] = {"config": "M = 2048 bf16 tokens, Q8 g32 / Q4 g64 weights, tcgen05 (fp16 operands, fp32 TMEM "
                                "accumulators); includes the activation tile prep", "peak_tflops": peak_t,
                      "peak_source": peaks["source"] + " (bf16 burst)", "cases": pre}
    ctx.close()
    torch.cuda.empty_cache()
    return out


# ----------------------------------------------------------------------------
# single GEMV workload
# ----------------------------------------------------------------------------

class GemvCase:
    """One quantized GEMV y[M, N] = x[M, K] . dequant(W)^T, seeded.
      8-bit : int8 codes U[-127, 127], fp16 scale per 32 columns,
              scales 0.02/127 * exp(N(0, 0.25))
      4/2-bit: unsigned codes packed little-endian (uniform), fp16 scale and
              zero per 64 columns, scales like those of quantized N(0, 0.02)
              weights, zeros in the middle of the code range
    x is N(0, 1) in fp32 or bf16."""

    def __init__(self, bits=8, N=12288, K=4096, M=1, xdtype="f32", seed=0):
        from chpe_qwen35_hybrid_engine_b200 import SCHEME_I8_GROUP_F16, SCHEME_U_GROUP_F16_ZERO
        self.bits, self.N, self.K, self.M, self.xdtype = bits, N, K, M, xdtype
        rng = np.random.default_rng(seed)
        if bits == 8:
            self.group, self.scheme = 32, SCHEME_I8_GROUP_F16
            self.codes = rng.integers(-127, 128, (N, K), dtype=np.int8)
            self.scales = (0.02 / 127 * np.exp(rng.normal(0, 0.25, (N, K // 32)))).astype(np.float16)
            self.zeros = None
        else:
            self.group, self.scheme = 64, SCHEME_U_GROUP_F16_ZERO
            self.codes = rng.integers(0, 256, (N, K * bits // 8), dtype=np.uint8)  # packed, uniform codes
            base = 0.02 * 5.0 / ((1 << bits) - 1)
            self.scales = (base * np.exp(rng.normal(0, 0.25, (N, K // 64)))).astype(np.float16)
            mid = (1 << bits) // 2
            self.zeros = rng.integers(mid - 2 if bits == 4 else 1, mid + 2 if bits == 4 else 3,
                                      (N, K // 64)).astype(np.float16)
        self.x = rng.standard_normal((M, K)).astype(np.float32)
        self.meta_bytes = self.scales.nbytes + (self.zeros.nbytes if self.zeros is not None else 0)

    @property
    def weight_bytes(self):
        return self.codes.nbytes + self.meta_bytes

    def algo_bytes(self):
        xb = 4 if self.xdtype == "f32" else 2
        return self.weight_bytes + self.M * self.K * xb + self.M * self.N * 4

    def unpacked(self):
        """Codes one per byte (for the oracle)."""
        if self.bits == 8:
            return self.codes
        per = 8 // self.bits
        out = np.empty((self.N, self.K), np.uint8)
        for j in range(per):
            out[:, j::per] = (self.codes >> (self.bits * j)) & ((1 << self.bits) - 1)
        return out

    def describe(self):
        return {"workload": "gemv", "bits": self.bits, "N": self.N, "K": self.K, "M": self.M, "group": self.group,
                "x": self.xdtype}


def gemv_metric(c):
    return (f"quantized GEMV HBM GB/s ({c.bits}-bit, group {c.group}, {c.N}x{c.K}, batch {c.M}, "
            f"{c.xdtype} activations)")


def run_gemv(args, rank, world, local_rank):
    import torch
    from chpe_qwen35_hybrid_engine_b200 import X_BF16, X_F32, Context
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    ctx = Context(local_rank)
    c = GemvCase(args.bits, args.rows, args.cols, args.batch, args.x)
    N, K, M = c.N, c.K, c.M
    algo = c.algo_bytes()
    n_copies = args.copies or max(2, int(np.ceil(3 * L2_BYTES / c.weight_bytes)))
    cd = torch.from_numpy(c.codes).to(dev)
    sd = torch.from_numpy(c.scales).to(dev)
    zd = torch.from_numpy(c.zeros).to(dev) if c.zeros is not None else None
    tens = [ctx.upload_matrix(c.bits, c.scheme, cd, sd, zd, rows=N, cols=K, group=c.group) for _ in range(n_copies)]
    del cd, sd, zd
    xdt = X_F32 if c.xdtype == "f32" else X_BF16
    xd = torch.from_numpy(c.x).to(dev)
    if c.xdtype == "bf16":
        xd = xd.to(torch.bfloat16)
    yd = torch.empty((M, N), dtype=torch.float32, device=dev)
    st = torch.cuda.Stream(dev)
    st.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(st):
        for i in range(args.warmup):
            ctx.gemv(tens[i % n_copies], xd, out=yd, stream=st)
    torch.cuda.synchronize(dev)
    clk = ClockSampler(local_rank).start()
    # a step = activation prep + GEMV through the public call; the K steps run as one graph
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=st):
        for i in range(args.steps):
            ctx.gemv(tens[i % n_copies], xd, out=yd, stream=st)
    graph.replay()
    ms_step = timed_replays(graph.replay, 1, world, dev) / args.steps
    del graph
    # the GEMV kernel alone (fragments prepared once)
    xf = ctx.xfrag(tens[0], M, xdt)
    ctx.xfrag_fill(xf, xd, stream=st)
    kgraph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(kgraph, stream=st):
        for i in range(args.steps):
            ctx.gemv_xfrag(tens[i % n_copies], xf, yd, stream=st)
    kgraph.replay()
    kern_ms = timed_replays(kgraph.replay, 3, 1, dev) / (3 * args.steps)
    del kgraph
    xf.free()
    # end to end through the public call, host buffers in pinned memory
    xh = xd.cpu().pin_memory()
    yh = torch.empty((M, N), dtype=torch.float32).pin_memory()
    xd2 = torch.empty_like(xd)
    rst = torch.cuda.current_stream(dev)
    it = [0]

    def e2e_step():
        xd2.copy_(xh, non_blocking=True)
        ctx.gemv(tens[it[0] % n_copies], xd2, out=yd, stream=rst)
        yh.copy_(yd, non_blocking=True)
        it[0] += 1

    for _ in range(args.warmup):
        e2e_step()
    e2e_ms = timed_replays(e2e_step, args.steps, world, dev) / args.steps
    clk.stop()
    peaks = measured_peaks()
    achieved = algo / (kern_ms * 1e-3) / 1e9
    cfg = c.describe()
    cfg.update({"l2": f"weights rotate over {n_copies} copies "
                      f"({n_copies * c.weight_bytes / 2**20:.0f} MiB > 2x L2)", "parallelism": f"replicas{world}"})
    line = {
        "metric": gemv_metric(c), "value": round(world * algo / (ms_step * 1e-3) / 1e9, 2), "unit": "GB/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms_step, 6),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": f"int{c.bits} codes x {c.xdtype} activations (fp16 tensor-core operands, fp32 accumulate)",
        "data": "synthetic (seeded uniform codes, lognormal fp16 group scales, x N(0,1))",
        "config": cfg,
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
                     "frac": round(achieved / peaks["hbm_gbs"], 4),
                     "traffic": NCU_TRAFFIC.get(("gemv", c.bits, N, K, M, c.xdtype)),
                     "peak_source": peaks["source"], "kernel": "chpe_qgemv_kernel", "kernel_us": round(kern_ms * 1e3, 3),
                     "algorithmic_bytes": algo},
        "e2e": {"value": round(world * algo / (e2e_ms * 1e-3) / 1e9, 2), "unit": "GB/s",
                "h2d_bytes_per_step": int(xd.numel() * xd.element_size()), "d2h_bytes_per_step": int(M * N * 4)},
        "gpu_launches": 2 * args.steps,
        "clocks": clk.summary(),
    }
    if rank == 0 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline_gemv(c)
    ctx.close()
    return line


def run_prefill(args, rank, world, local_rank):
    """Prefill dequant-GEMM: y[M, N] = x[M, K] . dequant(W)^T on tcgen05 (bf16
    activations N(0,1), the GemvCase weight formats); metric TFLOP/s."""
    import torch
    from chpe_qwen35_hybrid_engine_b200 import Context
    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    ctx = Context(local_rank)
    c = GemvCase(args.bits, args.rows, args.cols, 1, "bf16")
    N, K, M = c.N, c.K, args.batch
    flops = 2.0 * M * N * K
    cd = torch.from_numpy(c.codes).to(dev)
    sd = torch.from_numpy(c.scales).to(dev)
    zd = torch.from_numpy(c.zeros).to(dev) if c.zeros is not None else None
    n_copies = args.copies or max(2, int(np.ceil(3 * L2_BYTES / c.weight_bytes)))
    tens = [ctx.upload_matrix(c.bits, c.scheme, cd, sd, zd, rows=N, cols=K, group=c.group) for _ in range(n_copies)]
    del cd, sd, zd
    gen = torch.Generator(device=dev)
    gen.manual_seed(0)
    xd = torch.randn(M, K, device=dev, generator=gen).to(torch.bfloat16)
    yd = torch.empty(M, N, device=dev)
    st = torch.cuda.Stream(dev)
    st.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(st):
        for i in range(args.warmup):
            ctx.gemm_prefill(tens[i % n_copies], xd, out=yd, stream=st)
    torch.cuda.synchronize(dev)
    clk = ClockSampler(local_rank).start()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=st):
        for i in range(args.steps):
            ctx.gemm_prefill(tens[i % n_copies], xd, out=yd, stream=st)
    graph.replay()
    ms_step = timed_replays(graph.replay, 1, world, dev) / args.steps
    del graph
    # end to end: x from pinned host memory, y back to the host
    xh = xd.cpu().pin_memory()
    yh = torch.empty(M, N).pin_memory()
    xd2 = torch.empty_like(xd)
    rst = torch.cuda.current_stream(dev)
    it = [0]

    def e2e_step():
        xd2.copy_(xh, non_blocking=True)
        ctx.gemm_prefill(tens[it[0] % n_copies], xd2, out=yd, stream=rst)
        yh.copy_(yd, non_blocking=True)
        it[0] += 1

    for _ in range(args.warmup):
        e2e_step()
    e2e_ms = timed_replays(e2e_step, args.steps, world, dev) / args.steps
    clk.stop()
    ctx.sync()
    peaks = measured_peaks()
    tflops = flops / (ms_step * 1e-3) / 1e12
    peak = peaks["bf16_tflops"]
    cfg = {"workload": "prefill", "bits": c.bits, "N": N, "K": K, "M": M, "group": c.group, "x": "bf16",
           "l2": f"weights rotate over {n_copies} copies", "parallelism": f"replicas{world}"}
    line = {
        "metric": f"prefill dequant-GEMM TFLOP/s ({c.bits}-bit g{c.group}, M={M}, K={K}, N={N})",
        "value": round(world * tflops, 2), "unit": "TFLOP/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(ms_step, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "fp16 tensor-core operands (bf16 x, dequantized weights), fp32 accumulate",
        "data": "synthetic (seeded uniform codes, lognormal fp16 group scales, x N(0,1))", "config": cfg,
        "roofline": {"bound": "tensor", "achieved": round(tflops, 1), "peak": peak, "unit": "TFLOP/s",
                     "frac": round(tflops / peak, 4), "traffic": NCU_TRAFFIC.get(("prefill", c.bits, N, K, M)),
                     "peak_source": peaks["source"] + " (bf16 burst)",
                     "kernel": "prefill_gemm_kernel (+ activation tile prep)", "flops_per_step": flops},
        "e2e": {"value": round(world * flops / (e2e_ms * 1e-3) / 1e12, 2), "unit": "TFLOP/s",
                "h2d_bytes_per_step": int(M * K * 2), "d2h_bytes_per_step": int(M * N * 4)},
        "gpu_launches": 2 * args.steps,
        "clocks": clk.summary(),
    }
    ctx.close()
    return line


# ----------------------------------------------------------------------------
# CPU baselines: the oracle's C restatement of the reference path, host cores
# ----------------------------------------------------------------------------

def cpu_gemv_seconds(c, threads, reps=None, budget_s=10.0):
    from oracle import oracle as O
    codes = c.unpacked()
    O.gemv_grouped(codes, c.scales, c.zeros, c.group, c.x, num_workers=threads)  # warm-up
    t0 = time.perf_counter()
    n = 0
    while (reps is None and time.perf_counter() - t0 < budget_s) or (reps is not None and n < reps):
        O.gemv_grouped(codes, c.scales, c.zeros, c.group, c.x, num_workers=threads)
        n += 1
    return (time.perf_counter() - t0) / max(n, 1), n


def cpu_baseline_gemv(c, budget_s=10.0):
    threads = os.cpu_count() or 1
    dt, n = cpu_gemv_seconds(c, threads, budget_s=budget_s)
    return {"value": round(c.algo_bytes() / dt / 1e9, 3), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"{n} full {c.N}x{c.K} GEMVs at batch {c.M} by the C oracle (fp64 accumulation), "
                      f"{threads} threads"}


def cpu_decode_baseline(which, budget_s=12.0):
    """The reference engine's CPU decode step (oracle/cpu_baseline.c: the
    src/engine.zig worker pool and row split, the x86 int8 kernels for the 9B
    shape, the dotTileRow4Bit fp32 loop for the 4-bit 72B shape), whole steps,
    with every host thread and with the reference's NUM_WORKERS = 8
    (src/engine.zig:92)."""
    from oracle import cpu_baseline as CB
    nproc = os.cpu_count() or 1
    res = {}
    for th in sorted({nproc, 8}, reverse=True):
        tok_s, n, desc = CB.sample(which, th, budget_s=budget_s / 2, min_steps=2)
        res[th] = (tok_s, n, desc)
    tok_s, n, desc = res[nproc]
    return {"value": round(tok_s, 4), "unit": "tokens/s", "cores": nproc, "kind": "port", "sample": desc,
            "cpu_model": CB.cpu_model(),
            "by_threads": {str(t): {"tokens_s": round(v[0], 4), "steps": v[1]} for t, v in res.items()}}


def run_reference(args, rank, world, workload):
    """Reference arm on rank 0 (other ranks do nothing): the reference's CPU
    path with every host thread -- for the decode workloads the engine step
    restated in C (oracle/cpu_baseline.c), whole steps; for the single GEMV /
    prefill the oracle's grouped specification.  The Zig reference itself
    needs a Zig 0.17-dev toolchain absent from this image."""
    if rank != 0:
        return None
    threads = os.cpu_count() or 1
    if workload == "prefill":
        # a bounded sample: 8 activation rows through the oracle, scaled to M rows
        c = GemvCase(args.bits, args.rows, args.cols, 8, "bf16")
        for _ in range(args.warmup):
            cpu_gemv_seconds(c, threads, reps=1)
        dt, _ = cpu_gemv_seconds(c, threads, reps=args.steps)
        step = dt * args.batch / 8
        flops = 2.0 * args.batch * c.N * c.K
        value, unit, ms = round(flops / step / 1e12, 5), "TFLOP/s", step * 1e3
        metric = f"prefill dequant-GEMM TFLOP/s ({c.bits}-bit g{c.group}, M={args.batch}, K={c.K}, N={c.N})"
        sample = f"8 of {args.batch} activation rows per step through the C oracle (fp64 accumulation), scaled"
        cfg = {"workload": "prefill", "bits": c.bits, "N": c.N, "K": c.K, "M": args.batch, "group": c.group, "x": "bf16"}
        scaling = "weak"
    elif workload == "gemv":
        c = GemvCase(args.bits, args.rows, args.cols, args.batch, args.x)
        for _ in range(args.warmup):
            cpu_gemv_seconds(c, threads, reps=1)
        dt, _ = cpu_gemv_seconds(c, threads, reps=args.steps)
        value, unit, metric, ms = round(c.algo_bytes() / dt / 1e9, 3), "GB/s", gemv_metric(c), dt * 1e3
        sample = f"one full {c.N}x{c.K} GEMV at batch {c.M} per step (C oracle, fp64 accumulation)"
        cfg = c.describe()
        scaling = "weak"
    else:
        from oracle import cpu_baseline as CB
        d = CB.CpuDecoder(workload, threads)
        try:
            for _ in range(min(args.warmup, 2)):  # the host needs no more than a step to warm up
                d.step()
            est = [d.step() for _ in range(args.steps)]
            sample = d.describe(args.steps) + f"; model built in {d.build_s:.1f} s"
        finally:
            d.close()
        step = statistics.mean(est)
        value, unit, metric, ms = round(1.0 / step, 4), "tokens/s", DECODE_METRIC, step * 1e3
        cfg = decode_config(workload, world)
        scaling = "strong" if workload == "decode_72b" else "weak"
    return {"impl": "reference", "metric": metric, "value": value, "unit": unit, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
            "scaling": scaling, "vs_baseline": None,
            "dtype": "int codes; W8A8 int32 dots (9B) / fp32 4-bit loop (72B) / fp64 grouped spec (gemv, prefill)",
            "data": "synthetic (seeded)", "config": cfg,
            "cpu_baseline": {"value": value, "unit": unit, "cores": threads, "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="decode_72b", choices=["decode_72b", "decode_9b", "gemv", "q8_gemv", "prefill"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-sweep", action="store_true", help="decode: skip the single-kernel configurations at N = 1")
    ap.add_argument("--exchange", default="fill", choices=["fill", "push"],
                    help="decode_72b, N > 1: the O / down partials are sent by the fill that sums them (fill) "
                         "or by the GEMV that makes them (push)")
    ap.add_argument("--context", type=int, default=None,
                    help="decode: context tokens prefilled before the timed steps (default 1024 for 72B, 512 for 9B)")
    ap.add_argument("--bits", type=int, default=8, choices=[8, 4, 2], help="gemv: code width")
    ap.add_argument("--rows", type=int, default=12288, help="gemv: N (output columns)")
    ap.add_argument("--cols", type=int, default=4096, help="gemv: K (reduction length)")
    ap.add_argument("--batch", type=int, default=1, help="gemv: M (activation rows, 1..8); prefill: M")
    ap.add_argument("--x", default="f32", choices=["f32", "bf16"], help="gemv: activation dtype")
    ap.add_argument("--copies", type=int, default=0, help="gemv: weight copies to rotate (default: > 3x L2)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.workload == "q8_gemv":  # the single Q8 GEMV: 12288x4096, group 32, batch 1, fp32 x
        args.workload, args.bits, args.rows, args.cols, args.batch, args.x = "gemv", 8, 12288, 4096, 1, "f32"

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        line = run_reference(args, rank, world, args.workload)
        if line is not None:
            print(json.dumps(line), flush=True)
        return 0

    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                device_id=torch.device("cuda", local_rank))
    if args.workload == "gemv":
        line = run_gemv(args, rank, world, local_rank)
    elif args.workload == "prefill":
        line = run_prefill(args, rank, world, local_rank)
    else:
        line = run_decode(args, rank, world, local_rank, args.workload)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
