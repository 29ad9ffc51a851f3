"""ctypes front-end of oracle/cpu_baseline.c: the reference engine's CPU decode
step (src/engine.zig:583-734 with its x86 int8 kernels; the 4-bit
dotTileRow4Bit loop of src/qwen72b_engine.zig:135-148 for the 72B shape),
timed on whole steps on the host's cores.

TEST INFRASTRUCTURE ONLY: bench.py's cpu_baseline leg and its reference arm.
The library is compiled on the machine that runs it (-O3 -march=native, as the
reference's ReleaseFast build targets its host), into oracle/_cpu/.
"""
from __future__ import annotations

import ctypes as C
import hashlib
import os
import platform
import subprocess
import time

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_cpu")
_lib = None


def cpu_model() -> str:
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return platform.processor() or "unknown"


def mem_available_bytes() -> int:
    try:
        for line in open("/proc/meminfo"):
            if line.startswith("MemAvailable:"):
                return int(line.split()[1]) * 1024
    except OSError:
        pass
    return 16 << 30


def _key() -> str:
    flags = ""
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("flags"):
                flags = line
                break
    except OSError:
        pass
    src = open(os.path.join(HERE, "cpu_baseline.c"), "rb").read()
    return hashlib.sha1((cpu_model() + flags).encode() + src).hexdigest()[:12]


def lib():
    global _lib
    if _lib is not None:
        return _lib
    os.makedirs(OUT, exist_ok=True)
    so = os.path.join(OUT, f"libcpubaseline-{_key()}.so")
    if not os.path.exists(so):
        tmp = so + f".{os.getpid()}.tmp"
        subprocess.check_call(["gcc", "-O3", "-march=native", "-fPIC", "-shared", "-pthread", "-std=gnu11",
                               os.path.join(HERE, "cpu_baseline.c"), "-o", tmp, "-lm"])
        os.replace(tmp, so)
    L = C.CDLL(so)
    P, I, U64 = C.c_void_p, C.c_int, C.c_uint64
    L.cb_pool_create.restype, L.cb_pool_create.argtypes = P, [I]
    L.cb_pool_destroy.restype, L.cb_pool_destroy.argtypes = None, [P]
    L.cb_model_create.restype = P
    L.cb_model_create.argtypes = [P, I, I, I, I, I, I, I, I, I, I, I, I, U64]
    L.cb_model_destroy.restype, L.cb_model_destroy.argtypes = None, [P]
    L.cb_step.restype, L.cb_step.argtypes = I, [P, P, I]
    _lib = L
    return L


# (q4, n_layers, attn_every, hidden, ffn, vocab, q_dim, kv_dim, ssm_qkv, ssm_z, head_dim, bytes per layer)
SHAPES = {
    "decode_9b": (0, 32, 4, 4096, 12288, 151936, 8192, 1024, 6144, 2048, 256, 210 << 20),
    "decode_72b": (1, 80, 1, 8192, 29568, 152064, 8192, 1024, 0, 0, 128, 440 << 20),
}


class CpuDecoder:
    """One model of a benchmark shape on the host, stepping with `threads` workers."""

    def __init__(self, which: str, threads: int, seed: int = 0):
        L = lib()
        q4, nl, ae, H, F, V, qd, kd, sq, sz, hd, per_layer = SHAPES[which]
        # every layer gets its own weights when host memory allows, else they are reused in turn
        avail = mem_available_bytes() - (12 << 30)
        self.distinct = max(1, min(nl, avail // per_layer))
        self.threads = threads
        self.which = which
        self.pool = L.cb_pool_create(threads)
        t0 = time.perf_counter()
        self.m = L.cb_model_create(self.pool, q4, nl, ae, H, F, V, qd, kd, sq, sz, hd, int(self.distinct), seed)
        self.build_s = time.perf_counter() - t0
        if not self.m:
            L.cb_pool_destroy(self.pool)
            raise MemoryError("host memory for the CPU model")
        self.n_layers = nl
        self.tok = 17

    def step(self) -> float:
        """One whole decode step; returns its seconds."""
        t0 = time.perf_counter()
        self.tok = lib().cb_step(self.m, self.pool, self.tok)
        return time.perf_counter() - t0

    def describe(self, n: int) -> str:
        share = "" if self.distinct == self.n_layers else (
            f"; host memory held {self.distinct} layers' weights, reused in turn for the {self.n_layers}")
        kern = ("int8 W8A8 dots (x86 16-lane int32) and fused gate/up SwiGLU" if self.which == "decode_9b"
                else "4-bit dotTileRow4Bit fp32 loop (fp16 scale + zero per 64)")
        return (f"{n} whole decode steps of the reference engine's CPU path restated in C ({kern}, row split over "
                f"{self.threads} workers, src/engine.zig:94-313){share}; CPU {cpu_model()}")

    def close(self):
        if self.m:
            lib().cb_model_destroy(self.m)
            self.m = None
        if self.pool:
            lib().cb_pool_destroy(self.pool)
            self.pool = None


def sample(which: str, threads: int, budget_s: float = 10.0, min_steps: int = 2, max_steps: int = 50):
    """Whole-step tokens/s over a bounded sample (at least min_steps steps, then
    until budget_s has passed).  Returns (tokens/s, steps, description)."""
    d = CpuDecoder(which, threads)
    try:
        d.step()  # warm-up
        ts = []
        t0 = time.perf_counter()
        while len(ts) < min_steps or (time.perf_counter() - t0 < budget_s and len(ts) < max_steps):
            ts.append(d.step())
        return len(ts) / sum(ts), len(ts), d.describe(len(ts))
    finally:
        d.close()
