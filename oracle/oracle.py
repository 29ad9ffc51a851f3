"""ctypes/numpy front-end for the C oracle (oracle/chpe_oracle.c).

TEST INFRASTRUCTURE ONLY.  The oracle is the CPU restatement of the reference
CHPE hot path that the CUDA library is checked against.  Only tests/,
__graft_entry__.smoke() and bench.py's CPU-baseline leg import this module; the
product package never does.

Each wrapper names the reference function it restates (file:line inside the
reference project).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")
_lib = None


def build(force: bool = False) -> str:
    """Compile oracle/chpe_oracle.c into oracle/liboracle.so with gcc."""
    src = os.path.join(_HERE, "chpe_oracle.c")
    if force or not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(src):
        subprocess.check_call(["make", "-s", "-C", _HERE])
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        build()
        _lib = C.CDLL(_LIB_PATH)
        _declare(_lib)
    return _lib


P = C.c_void_p
SZ = C.c_size_t
F = C.c_float
I = C.c_int


def _declare(L):
    sigs = {
        "oracle_dot_i8": (F, [P, P, SZ, F, F]),
        "oracle_dot_i8_quadrow": (None, [P, P, P, P, P, SZ, F, F, P]),
        "oracle_dot_i8_gateup_swiglu": (F, [P, P, P, SZ, F, F, F]),
        "oracle_dot_i8_batch": (None, [P, P, I, SZ, F, P, P]),
        "oracle_quantize_act_i8": (F, [P, SZ, P]),
        "oracle_rmsnorm": (None, [P, P, P, SZ, F]),
        "oracle_silu_mul": (None, [P, P, P, SZ]),
        "oracle_gemv_parallel": (None, [P, F, P, F, SZ, SZ, P, I]),
        "oracle_gemv_gateup_swiglu_parallel": (None, [P, F, P, F, P, F, SZ, SZ, P, I]),
        "oracle_gemv_batch_parallel": (None, [P, F, P, P, I, SZ, SZ, P, I]),
        "oracle_gemv_tile_w2": (None, [P, P, SZ, P, SZ, I]),
        "oracle_gemv_tile_w4": (None, [P, P, P, SZ, I]),
        "oracle_gemv_tile_w8": (None, [P, P, P, SZ, I]),
        "oracle_gemv_tile_polymorphic": (None, [P, P, SZ, P, SZ, I]),
        "oracle_dot_tile_row_2bit": (F, [P, P, SZ, F, F]),
        "oracle_dot_tile_row_4bit": (F, [P, P, SZ, F, F]),
        "oracle_quantize_4bit_block": (None, [P, SZ, P, P]),
        "oracle_quantize_2bit_block": (None, [P, SZ, P, P]),
        "oracle_quantize_asym": (None, [P, SZ, SZ, I, I, P, P, P]),
        "oracle_quantize_sym8": (None, [P, SZ, SZ, I, P, P]),
        "oracle_gemv_grouped": (None, [I, P, P, P, I, SZ, SZ, P, I, SZ, P]),
        "oracle_gemv_grouped_mt": (None, [I, P, P, P, I, SZ, SZ, P, I, SZ, P, I]),
        "oracle_argmax": (C.c_uint32, [P, SZ, P]),
    }
    for name, (res, args) in sigs.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args


def _p(a: np.ndarray):
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(C.c_void_p)


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


# --- src/kernels/neon.zig ---------------------------------------------------

def dot_i8(a, b, scale_w, scale_x):
    """src/kernels/neon.zig:54-124 dotProductInt8Neon."""
    a, b = _c(a, np.int8), _c(b, np.int8)
    return lib().oracle_dot_i8(_p(a), _p(b), a.size, scale_w, scale_x)


def dot_i8_quadrow(w4, x, scale_w, scale_x):
    """src/kernels/neon.zig:129-255 dotProductInt8QuadRowNeon; w4 is [4, n]."""
    w4, x = _c(w4, np.int8), _c(x, np.int8)
    out = np.zeros(4, np.float32)
    lib().oracle_dot_i8_quadrow(_p(w4[0]), _p(w4[1]), _p(w4[2]), _p(w4[3]), _p(x), x.size, scale_w, scale_x, _p(out))
    return out


def dot_i8_gateup_swiglu(wg, wu, x, sg, su, sx):
    """src/kernels/neon.zig:261-350 dotProductInt8GateUpSwiGLUNeon."""
    wg, wu, x = _c(wg, np.int8), _c(wu, np.int8), _c(x, np.int8)
    return lib().oracle_dot_i8_gateup_swiglu(_p(wg), _p(wu), _p(x), x.size, sg, su, sx)


def dot_i8_batch(w, xs, scale_w, scales_x):
    """src/kernels/neon.zig:355-641 dotProductInt8Batch4Neon / Batch8Neon; xs is [nb, n]."""
    w, xs = _c(w, np.int8), _c(xs, np.int8)
    sxs = _c(scales_x, np.float32)
    nb = xs.shape[0]
    ptrs = (C.c_void_p * nb)(*[xs[b].ctypes.data for b in range(nb)])
    out = np.zeros(nb, np.float32)
    lib().oracle_dot_i8_batch(_p(w), C.cast(ptrs, C.c_void_p), nb, w.size, scale_w, _p(sxs), _p(out))
    return out


def quantize_act_i8(x):
    """src/kernels/neon.zig:644-670 quantizeActivationInt8 -> (q int8, scale)."""
    x = _c(x, np.float32)
    q = np.zeros(x.size, np.int8)
    s = lib().oracle_quantize_act_i8(_p(x), x.size, _p(q))
    return q, np.float32(s)


def rmsnorm(x, gamma, eps=1e-6):
    """src/kernels/neon.zig:673-702 rmsnorm."""
    x, gamma = _c(x, np.float32), _c(gamma, np.float32)
    y = np.zeros_like(x)
    lib().oracle_rmsnorm(_p(x), _p(gamma), _p(y), x.size, eps)
    return y


def silu_mul(g, u):
    """src/kernels/neon.zig:705-712 siluMul."""
    g, u = _c(g, np.float32), _c(u, np.float32)
    out = np.zeros_like(g)
    lib().oracle_silu_mul(_p(g), _p(u), _p(out), g.size)
    return out


# --- src/engine.zig GEMV operators -------------------------------------------

def gemv_parallel(weights, scale_w, x_q8, scale_x, num_workers=8):
    """src/engine.zig:227-251 gemvParallel; weights is [rows, cols] int8."""
    w = _c(weights, np.int8)
    x = _c(x_q8, np.int8)
    rows, cols = w.shape
    out = np.zeros(rows, np.float32)
    lib().oracle_gemv_parallel(_p(w), scale_w, _p(x), scale_x, rows, cols, _p(out), num_workers)
    return out


def gemv_gateup_swiglu_parallel(gate, scale_gate, up, scale_up, x_q8, scale_x, num_workers=8):
    """src/engine.zig:285-313 gemvGateUpSwiGLUParallel."""
    g, u, x = _c(gate, np.int8), _c(up, np.int8), _c(x_q8, np.int8)
    rows, cols = g.shape
    out = np.zeros(rows, np.float32)
    lib().oracle_gemv_gateup_swiglu_parallel(_p(g), scale_gate, _p(u), scale_up, _p(x), scale_x, rows, cols,
                                             _p(out), num_workers)
    return out


def gemv_batch_parallel(weights, scale_w, xs_q8, scales_x, num_workers=8):
    """src/engine.zig:357-391 gemvBatch4Parallel / :434-460 gemvBatch8Parallel.
    xs_q8 is [nb, cols]; returns [nb, rows]."""
    w = _c(weights, np.int8)
    xs = _c(xs_q8, np.int8)
    sxs = _c(scales_x, np.float32)
    rows, cols = w.shape
    nb = xs.shape[0]
    outs = np.zeros((nb, rows), np.float32)
    xp = (C.c_void_p * nb)(*[xs[b].ctypes.data for b in range(nb)])
    op = (C.c_void_p * nb)(*[outs[b].ctypes.data for b in range(nb)])
    lib().oracle_gemv_batch_parallel(_p(w), scale_w, C.cast(xp, C.c_void_p), _p(sxs), nb, rows, cols,
                                     C.cast(op, C.c_void_p), num_workers)
    return outs


# --- src/chpe_engine.zig / src/qwen72b_engine.zig tile GEMVs -----------------

def gemv_tile_polymorphic(cell: np.ndarray, x, y=None, row_base=0, accumulate=False):
    """src/chpe_engine.zig:469-488 gemvTilePolymorphic over one 17408-byte cell."""
    cell = _c(cell, np.uint8)
    assert cell.size == 17408
    x = _c(x, np.float32)
    if y is None:
        rows = int(np.frombuffer(cell[16448 + 40:16448 + 44].tobytes(), np.uint32)[0])
        y = np.zeros(row_base + rows, np.float32)
    lib().oracle_gemv_tile_polymorphic(_p(cell), _p(x), x.size, _p(y), row_base, int(accumulate))
    return y


def dot_tile_row_2bit(coded, x, scale, bias):
    """src/qwen72b_engine.zig:119-132 dotTileRow2Bit."""
    coded, x = _c(coded, np.uint8), _c(x, np.float32)
    return lib().oracle_dot_tile_row_2bit(_p(coded), _p(x), x.size, scale, bias)


def dot_tile_row_4bit(coded, x, scale, bias):
    """src/qwen72b_engine.zig:135-148 dotTileRow4Bit."""
    coded, x = _c(coded, np.uint8), _c(x, np.float32)
    return lib().oracle_dot_tile_row_4bit(_p(coded), _p(x), x.size, scale, bias)


# --- quantizers ---------------------------------------------------------------

def quantize_4bit_block(blk):
    """scripts/pack_qwen72b_chpe.py:138-148; blk [N,128] f32 -> (packed u8 [N*64], scales f16 [N])."""
    blk = _c(blk, np.float32).reshape(-1, 128)
    n = blk.shape[0]
    packed = np.zeros(n * 64, np.uint8)
    scales = np.zeros(n, np.uint16)
    lib().oracle_quantize_4bit_block(_p(blk), n, _p(packed), _p(scales))
    return packed, scales.view(np.float16)


def quantize_2bit_block(blk):
    """scripts/pack_qwen72b_chpe.py:110-135; blk [N,128] f32 -> (packed u8 [N*32], scales f16 [N])."""
    blk = _c(blk, np.float32).reshape(-1, 128)
    n = blk.shape[0]
    packed = np.zeros(n * 32, np.uint8)
    scales = np.zeros(n, np.uint16)
    lib().oracle_quantize_2bit_block(_p(blk), n, _p(packed), _p(scales))
    return packed, scales.view(np.float16)


def quantize_asym(w, bits, group):
    """Unsigned codes + fp16 scale + fp16 zero per group (this project's spec)."""
    w = _c(w, np.float32)
    rows, cols = w.shape
    codes = np.zeros((rows, cols), np.uint8)
    s = np.zeros((rows, cols // group), np.uint16)
    z = np.zeros((rows, cols // group), np.uint16)
    lib().oracle_quantize_asym(_p(w), rows, cols, bits, group, _p(codes), _p(s), _p(z))
    return codes, s.view(np.float16), z.view(np.float16)


def quantize_sym8(w, group):
    """Signed int8 codes in [-127,127] + fp16 scale per group (this project's spec)."""
    w = _c(w, np.float32)
    rows, cols = w.shape
    codes = np.zeros((rows, cols), np.int8)
    s = np.zeros((rows, cols // group), np.uint16)
    lib().oracle_quantize_sym8(_p(w), rows, cols, group, _p(codes), _p(s))
    return codes, s.view(np.float16)


def gemv_grouped(codes, scales, zeros, group, x, num_workers=1):
    """Grouped dequant-GEMV specification, fp64 accumulation.
    codes [N,K] (int8 when zeros is None, else uint8); scales/zeros [N,K/group] f16;
    x [M,K] float32 or bf16 (given as uint16 bit patterns, dtype np.uint16)."""
    signed = zeros is None
    codes = _c(codes, np.int8 if signed else np.uint8)
    N, K = codes.shape
    sc = _c(np.asarray(scales, np.float16).view(np.uint16), np.uint16)
    zc = None if signed else _c(np.asarray(zeros, np.float16).view(np.uint16), np.uint16)
    if x.dtype == np.uint16:
        xk, xx = 1, _c(x, np.uint16)
    else:
        xk, xx = 0, _c(x, np.float32)
    xx = xx.reshape(-1, K)
    M = xx.shape[0]
    y = np.zeros((M, N), np.float32)
    lib().oracle_gemv_grouped_mt(int(signed), _p(codes), _p(sc), None if zc is None else _p(zc), group, N, K,
                                 _p(xx), xk, M, _p(y), num_workers)
    return y


def argmax(logits):
    """src/engine.zig:1098-1110 computeArgmax."""
    l = _c(logits, np.float32)
    mv = np.zeros(1, np.float32)
    i = lib().oracle_argmax(_p(l), l.size, _p(mv))
    return int(i), float(mv[0])
