"""CPU tests of the C ABI: the library builds for sm_100a, loads, and exports
every entry point include/chpe_b200.h declares.  No kernel is called."""
import ctypes
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER_DIR = os.path.join(ROOT, "include")


def declared_functions():
    names = set()
    for fn in os.listdir(HEADER_DIR):
        if not fn.endswith(".h"):
            continue
        src = open(os.path.join(HEADER_DIR, fn)).read()
        src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
        for m in re.finditer(r"\b(?:int|const char \*|void)\s*\**\s*(chpe_\w+)\s*\(", src):
            names.add(m.group(1))
    return names


def test_header_declares_entry_points():
    names = declared_functions()
    for required in ("chpe_init", "chpe_gemv_parallel", "chpe_gemv_gate_up_swiglu_parallel",
                     "chpe_gemv_batch4_parallel", "chpe_gemv_batch8_parallel", "chpe_quantize_activation_int8",
                     "chpe_gemv_tile_polymorphic", "chpe_gemv_dev", "chpe_upload_matrix", "chpe_upload_cells"):
        assert required in names


def test_library_exports_every_declared_symbol():
    from chpe_qwen35_hybrid_engine_b200 import _lib
    from chpe_qwen35_hybrid_engine_b200 import build
    build.build()
    lib = ctypes.CDLL(_lib.LIB_PATH)
    missing = [n for n in sorted(declared_functions()) if not hasattr(lib, n)]
    assert not missing, missing
    # the Python binding covers the same set
    assert declared_functions() <= set(_lib.SIGNATURES)


def test_binding_loads_and_reports_version():
    from chpe_qwen35_hybrid_engine_b200 import Context
    assert "sm_100a" in Context.version()


def test_init_without_gpu_fails_cleanly():
    import torch
    if torch.cuda.is_available():
        pytest.skip("GPU present")
    from chpe_qwen35_hybrid_engine_b200 import ChpeError, Context
    with pytest.raises(ChpeError):
        Context(0)


def test_product_does_not_reference_oracle():
    """The product package never imports or links the oracle."""
    pkg = os.path.join(ROOT, "chpe_qwen35_hybrid_engine_b200")
    for dirpath, _, files in os.walk(pkg):
        for f in files:
            if f.endswith((".py", ".cu", ".cuh", ".h", ".cpp")):
                txt = open(os.path.join(dirpath, f)).read()
                assert "oracle" not in txt.replace("the oracle", ""), f
