"""ctypes binding of libchpe_b200.so (include/chpe_b200.h).

Loading fails loudly when the shared library is missing: there is no CPU
fallback anywhere in this package.
"""
from __future__ import annotations

import ctypes as C
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libchpe_b200.so")

# status codes (include/chpe_b200.h)
OK, EINVAL, EALIGN, ENOMEM, ECUDA, ETIMEOUT, ENOTSUP, ENOENT = 0, -1, -2, -3, -4, -5, -6, -7
STATUS_NAMES = {0: "OK", -1: "EINVAL", -2: "EALIGN", -3: "ENOMEM", -4: "ECUDA", -5: "ETIMEOUT", -6: "ENOTSUP",
                -7: "ENOENT"}

SCHEME_I8_TENSOR = 1
SCHEME_I8_GROUP_F16 = 2
SCHEME_U_GROUP_F16_ZERO = 3
SCHEME_U_GROUP_F16_CONST_ZERO = 4
SCHEME_W2_CODEBOOK_GROUP_F16 = 5
SCHEME_ROW_AFFINE_F32 = 6

X_F32, X_BF16, X_F16, X_I8 = 0, 1, 2, 3

XOP_PLAIN, XOP_RMSNORM, XOP_SILU_MUL, XOP_ATTN_STUB, XOP_SSM_STUB = 0, 1, 2, 3, 4


class chpe_fmt(C.Structure):
    _fields_ = [("bits", C.c_int32), ("scheme", C.c_int32), ("group", C.c_int32), ("zero", C.c_float)]


class chpe_xsrc(C.Structure):
    _fields_ = [("op", C.c_int32), ("x", C.c_void_p), ("x_dtype", C.c_int32), ("ldx", C.c_int32),
                ("aux", C.c_void_p), ("ld_aux", C.c_int32), ("eps", C.c_float), ("kv_dim", C.c_int32),
                ("head_dim", C.c_int32), ("group", C.c_int32), ("qkv_dim", C.c_int32), ("silu_on_qkv", C.c_int32)]


P = C.c_void_p
SZ = C.c_size_t
I = C.c_int
F = C.c_float
PP = C.POINTER(C.c_void_p)

# name -> (restype, argtypes); every symbol declared in include/chpe_b200.h
SIGNATURES = {
    "chpe_init": (I, [I, PP]),
    "chpe_destroy": (I, [P]),
    "chpe_last_error_string": (C.c_char_p, [P]),
    "chpe_version": (C.c_char_p, []),
    "chpe_kernel_launches": (C.c_ulonglong, []),
    "chpe_sync": (I, [P]),
    "chpe_upload_matrix": (I, [P, C.POINTER(chpe_fmt), P, SZ, P, P, P, SZ, SZ, PP]),
    "chpe_upload_cells": (I, [P, P, SZ, SZ, PP]),
    "chpe_quantize_group_dev": (I, [P, P, SZ, SZ, I, I, I, P, P, P, P]),
    "chpe_tensor_free": (I, [P, P]),
    "chpe_tensor_info": (I, [P, C.POINTER(SZ), C.POINTER(SZ), C.POINTER(I), C.POINTER(SZ)]),
    "chpe_register_i8": (I, [P, P, SZ, SZ]),
    "chpe_tensor_unpack": (I, [P, P, P, P, P]),
    "chpe_gemv_dev": (I, [P, P, P, I, P, I, P, I, P]),
    "chpe_gemv_gateup_swiglu_dev": (I, [P, P, P, P, I, P, I, P, P]),
    "chpe_quantize_act_i8_dev": (I, [P, P, I, SZ, P, P, P]),
    "chpe_gemv_noalloc_dev": (I, [P, P, P, I, P, I, P, P]),
    "chpe_embed_i8_dev": (I, [P, P, F, I, I, P, I, P, P]),
    "chpe_rmsnorm_dev": (I, [P, P, P, I, I, F, P, P]),
    "chpe_mix_attn_stub_dev": (I, [P, P, I, I, I, I, I, P, P]),
    "chpe_mix_ssm_stub_dev": (I, [P, P, I, P, I, I, I, I, P, P]),
    "chpe_silu_mul_dev": (I, [P, P, P, SZ, P, P]),
    "chpe_argmax_dev": (I, [P, P, I, I, P, P, P]),
    "chpe_attn_decode_dev": (I, [P, P, I, P, P, I, P, P, P, I, I, I, I, I, F, I, P, I, P]),
    "chpe_deltanet_step_dev": (I, [P, P, I, P, P, P, P, P, I, I, I, I, P, I, P]),
    "chpe_pos_advance_dev": (I, [P, P, I, P]),
    "chpe_xfrag_create": (I, [P, P, I, I, PP]),
    "chpe_xfrag_fill_dev": (I, [P, P, P, P, P]),
    "chpe_gemv_xfrag_dev": (I, [P, P, P, P, I, P]),
    "chpe_gemv_gateup_swiglu_xfrag_dev": (I, [P, P, P, P, P, P]),
    "chpe_gemv_multi_xfrag_dev": (I, [P, I, P, P, P, P]),
    "chpe_gemm_prefill_dev": (I, [P, P, P, I, I, P, I, I, P]),
    "chpe_comm_create": (I, [P, I, I, SZ, PP]),
    "chpe_comm_handle_bytes": (SZ, []),
    "chpe_comm_handle": (I, [P, P]),
    "chpe_comm_open_peers": (I, [P, P]),
    "chpe_allreduce_residual_dev": (I, [P, P, P, SZ, P]),
    "chpe_argmax_merge_dev": (I, [P, P, P, I, I, P]),
    "chpe_allreduce_fill_dev": (I, [P, P, P, P, P, F, I, P]),
    "chpe_gemv_xfrag_push_dev": (I, [P, P, P, P, P, P]),
    "chpe_comm_failed": (I, [P]),
    "chpe_comm_reset": (I, [P]),
    "chpe_comm_destroy": (I, [P]),
    "chpe_xfrag_free": (I, [P, P]),
    "chpe_xfrag_fill_op_dev": (I, [P, P, C.POINTER(chpe_xsrc), P]),
    "chpe_gemv_src_dev": (I, [P, I, I, P, C.POINTER(chpe_xsrc), I, P, I, P]),
    "chpe_gemv_parallel": (I, [P, P, F, P, F, SZ, SZ, P]),
    "chpe_gemv_gate_up_swiglu_parallel": (I, [P, P, F, P, F, P, F, SZ, SZ, P]),
    "chpe_gemv_batch4_parallel": (I, [P, P, F, P, P, P, P, P, SZ, SZ, P, P, P, P]),
    "chpe_gemv_batch8_parallel": (I, [P, P, F, P, P, SZ, SZ, P]),
    "chpe_quantize_activation_int8": (I, [P, P, SZ, P, P]),
    "chpe_gemv_tile_polymorphic": (I, [P, P, P, SZ, P, SZ, I]),
}

_lib = None


class ChpeError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"{STATUS_NAMES.get(code, code)}: {msg}")
        self.code = code


def load(build_if_missing: bool = True):
    """Load libchpe_b200.so (building it first when absent and nvcc exists)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH) and build_if_missing:
        from . import build as _build
        _build.build()
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"CUDA library {LIB_PATH} is missing; run python -m chpe_qwen35_hybrid_engine_b200.build")
    lib = C.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib
