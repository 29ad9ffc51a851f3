"""Build the sm_100a shared library libchpe_b200.so in-tree with nvcc.

    python -m chpe_qwen35_hybrid_engine_b200.build [--force] [--verbose]

Each .cu under csrc/ is compiled to an object (parallel), then linked into
chpe_qwen35_hybrid_engine_b200/libchpe_b200.so.  Only sm_100a code is
generated (-gencode arch=compute_100a,code=sm_100a).
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OBJ = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libchpe_b200.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVFLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
           "--expt-relaxed-constexpr", "-I", os.path.join(ROOT, "include")]
SOURCES = ["gemv.cu", "gemv_b8.cu", "gemv_b4.cu", "gemv_b2.cu", "gemv_b2w.cu", "gemv_s8.cu", "prep.cu", "model.cu", "mixers.cu", "prefill.cu", "comm.cu", "abi.cu"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _deps_mtime() -> float:
    m = 0.0
    for d in (CSRC, os.path.join(ROOT, "include")):
        for f in os.listdir(d):
            m = max(m, os.path.getmtime(os.path.join(d, f)))
    return m


def needs_build() -> bool:
    return not os.path.exists(LIB) or os.path.getmtime(LIB) < _deps_mtime()


def build(force: bool = False, verbose: bool = False, extra: list[str] | None = None) -> str:
    if not force and not needs_build():
        return LIB
    os.makedirs(OBJ, exist_ok=True)
    cc = nvcc()
    extra = extra or []

    def compile_one(src: str) -> str:
        obj = os.path.join(OBJ, src.replace(".cu", ".o"))
        cmd = [cc, *ARCH, *NVFLAGS, *extra, "-c", os.path.join(CSRC, src), "-o", obj]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
        if verbose and (r.stdout or r.stderr):
            print(r.stdout, r.stderr, flush=True)
        return obj

    with cf.ThreadPoolExecutor(max_workers=len(SOURCES)) as ex:
        objs = list(ex.map(compile_one, SOURCES))
    tmp = LIB + ".tmp"
    cmd = [cc, *ARCH, "-shared", "-o", tmp, *objs, "-lcudart"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-v", action="store_true", help="print register / shared-memory usage")
    a = ap.parse_args()
    extra = ["-Xptxas", "-v"] if a.ptxas_v else []
    print(build(force=a.force or a.ptxas_v, verbose=a.verbose or a.ptxas_v, extra=extra))
    sys.exit(0)
