"""The allocation-free GEMV entry point (chpe_gemv_noalloc_dev).

Some callers cannot allocate device memory while they run a GEMV -- an engine
that reserved all its device memory once at start-up and treats any later
cudaMalloc as a failure, or a decode loop that cannot take cudaMalloc's
implicit device synchronisation.  This entry point keeps its scratch in a
static device array instead of the context's cudaMalloc'd scratch.  These
tests call it through the C ABI on a fresh context (whose own scratch was
never grown): after a first set-up call, the device's free memory must not
move across two more calls, and both calls must equal chpe_gemv_dev on the
same inputs bit for bit: the two run the same kernel and launch plan, so every format gives
identical bits, and the second call shows that nothing stale from the first
leaks through the shared array.  The file is named so pytest collects it last.
"""
import ctypes as C

import numpy as np
import pytest

from oracle import oracle as O
from tests._util import pack_codes, rel_l2

pytestmark = pytest.mark.gpu
TOL = 1e-3


def _noalloc(ctx, t, x, x_dtype, M, y, x_scales=None):
    import torch
    st = torch.cuda.current_stream()
    rc = ctx.lib.chpe_gemv_noalloc_dev(ctx.ptr, t.handle, C.c_void_p(x.data_ptr()), x_dtype,
                                       None if x_scales is None else C.c_void_p(x_scales.data_ptr()), M,
                                       C.c_void_p(y.data_ptr()), C.c_void_p(st.cuda_stream))
    return rc


@pytest.mark.parametrize("fmt", ["q4_g64_bf16_m4", "q8_g32_f32_m1", "w8a8_m8", "q2_g64_f32_m8"])
def test_noalloc_matches_gemv_dev_twice(fmt):
    import torch
    from chpe_qwen35_hybrid_engine_b200 import (SCHEME_I8_GROUP_F16, SCHEME_I8_TENSOR, SCHEME_U_GROUP_F16_ZERO,
                                                X_BF16, X_F32, X_I8, Context)
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    ctx = Context(0)  # fresh: its growable scratch has never been allocated
    rng = np.random.default_rng(42)
    if fmt == "q4_g64_bf16_m4":
        N, K, M = 3000, 4096, 4
        codes, s, z = O.quantize_asym(rng.normal(0, 0.02, (N, K)).astype(np.float32), 4, 64)
        t = ctx.upload_matrix(4, SCHEME_U_GROUP_F16_ZERO, pack_codes(codes, 4), s, z, rows=N, cols=K, group=64)
        xs = [torch.randn(M, K, device="cuda").to(torch.bfloat16) for _ in range(2)]
        dt, scales = X_BF16, None
    elif fmt == "q2_g64_f32_m8":
        N, K, M = 2048, 4096, 8
        codes, s, z = O.quantize_asym(rng.normal(0, 0.02, (N, K)).astype(np.float32), 2, 64)
        t = ctx.upload_matrix(2, SCHEME_U_GROUP_F16_ZERO, pack_codes(codes, 2), s, z, rows=N, cols=K, group=64)
        xs = [torch.randn(M, K, device="cuda") for _ in range(2)]
        dt, scales = X_F32, None
    elif fmt == "q8_g32_f32_m1":
        N, K, M = 12288, 4096, 1
        codes = rng.integers(-127, 128, (N, K), dtype=np.int8)
        s = (0.02 / 127 * np.exp(rng.normal(0, 0.25, (N, K // 32)))).astype(np.float16)
        t = ctx.upload_matrix(8, SCHEME_I8_GROUP_F16, codes, s, rows=N, cols=K, group=32)
        xs = [torch.randn(M, K, device="cuda") for _ in range(2)]
        dt, scales = X_F32, None
    else:
        N, K, M = 1000, 2048, 8
        w = rng.integers(-127, 128, (N, K), dtype=np.int8)
        t = ctx.upload_matrix(8, SCHEME_I8_TENSOR, w, np.array([0.003], np.float32), rows=N, cols=K)
        xs = [torch.randint(-128, 128, (M, K), dtype=torch.int8, device="cuda") for _ in range(2)]
        dt, scales = X_I8, torch.rand(M, device="cuda") * 0.05 + 0.001
    ys = [torch.full((M, N), float("nan"), device="cuda") for _ in range(2)]
    # set-up call: the first call on a device looks up the static array's
    # device address, and the CUDA runtime may load the library's module (and
    # with it the array, which it then holds until exit) only at that point
    assert _noalloc(ctx, t, xs[0], dt, M, ys[0], scales) == 0, ctx.lib.chpe_last_error_string(ctx.ptr)
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    for x, y in zip(xs, ys):  # two calls in a row, different activations
        assert _noalloc(ctx, t, x, dt, M, y, scales) == 0, ctx.lib.chpe_last_error_string(ctx.ptr)
        torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free0  # no device memory was allocated
    for x, y in zip(xs, ys):
        ref = ctx.gemv(t, x, x_scales=scales)
        torch.cuda.synchronize()
        assert torch.isfinite(y).all()
        assert rel_l2(y.cpu().numpy(), ref.cpu().numpy()) < TOL
        assert torch.equal(y, ref)  # same kernel, same plan: identical bits
    ctx.sync()
    t.free()
    ctx.close()


def test_noalloc_rejects_shapes_beyond_its_scratch(ctx):
    import torch
    from chpe_qwen35_hybrid_engine_b200 import SCHEME_U_GROUP_F16_ZERO, X_BF16
    N, K, M = 16, 1 << 21, 8  # the activation fragments alone (32 MiB) exceed the 16 MiB array
    t = ctx.upload_matrix(4, SCHEME_U_GROUP_F16_ZERO, np.zeros((N, K // 2), np.uint8),
                          np.ones((N, K // 64), np.float16), np.zeros((N, K // 64), np.float16), rows=N, cols=K,
                          group=64)
    x = torch.zeros(M, K, device="cuda", dtype=torch.bfloat16)
    y = torch.zeros(M, N, device="cuda")
    rc = _noalloc(ctx, t, x, X_BF16, M, y)
    assert rc == -1  # CHPE_EINVAL
    assert b"allocation-free GEMV has" in ctx.lib.chpe_last_error_string(ctx.ptr)
    rc = _noalloc(ctx, t, x, X_BF16, 9, y)
    assert rc == -1
    t.free()
