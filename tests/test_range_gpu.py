"""Activation range: rows far outside fp16's range through the GEMV and the
prefill GEMM.

Both paths feed the tensor cores fp16 activations (fp32 rows as an fp16 hi +
lo pair).  Every activation row is first scaled by a power of two chosen from
its largest magnitude, and the epilogue undoes it, so rows of 1e6 (above
fp16's 65504) and of 1e-30 (far below its smallest subnormal) keep the fp32
oracle's results: rel-L2 <= 1e-3 per row (the path's tolerance, TOL) with
finite outputs, for fp32 and bf16 activations, M = 1 and 8, the three code
widths, and prefill.  The oracle accumulates in fp64 on the unscaled inputs.
"""
import numpy as np
import pytest

from oracle import oracle as O
from tests._util import pack_codes, rel_l2

pytestmark = pytest.mark.gpu
TOL = 1e-3

MAGS = [1e6, 1e-30, 3e4, 1.0, 1e-6, 1e12, 2e-38, 7e-3]  # one magnitude per row


def _tensor(ctx, rng, bits, N, K):
    from chpe_qwen35_hybrid_engine_b200 import SCHEME_I8_GROUP_F16, SCHEME_U_GROUP_F16_ZERO
    w = rng.normal(0, 0.02, (N, K)).astype(np.float32)
    if bits == 8:
        codes, s = O.quantize_sym8(w, 32)
        t = ctx.upload_matrix(8, SCHEME_I8_GROUP_F16, codes, s, rows=N, cols=K, group=32)
        return t, (codes, s, None, 32)
    codes, s, z = O.quantize_asym(w, bits, 64)
    t = ctx.upload_matrix(bits, SCHEME_U_GROUP_F16_ZERO, pack_codes(codes, bits), s, z, rows=N, cols=K, group=64)
    return t, (codes, s, z, 64)


def _rows(rng, M, K, mags):
    x = rng.standard_normal((M, K)).astype(np.float64)
    for m in range(M):
        x[m] *= mags[m % len(mags)]
    return x.astype(np.float32)


def _check_rows(got, want):
    assert np.isfinite(got).all()
    for m in range(got.shape[0]):
        e = rel_l2(got[m], want[m])
        assert e < TOL, (m, e)


@pytest.mark.parametrize("bits", [8, 4, 2])
@pytest.mark.parametrize("M", [1, 8])
@pytest.mark.parametrize("xdt", ["f32", "bf16"])
def test_gemv_extreme_rows(ctx, bits, M, xdt):
    import torch
    rng = np.random.default_rng(bits * 100 + M + (7 if xdt == "bf16" else 0))
    N, K = 512, 4096
    t, (codes, s, z, group) = _tensor(ctx, rng, bits, N, K)
    for shift in range(0, 8 if M == 1 else 1):  # at M = 1 every magnitude in turn
        mags = MAGS[shift:] + MAGS[:shift]
        x = _rows(rng, M, K, mags)
        xd = torch.from_numpy(x).cuda()
        if xdt == "bf16":
            xd = xd.to(torch.bfloat16)
        y = ctx.gemv(t, xd)
        torch.cuda.synchronize()
        xo = xd.float().cpu().numpy()  # the values the kernel was given
        want = O.gemv_grouped(codes, s, z, group, xo, num_workers=8)
        _check_rows(y.cpu().numpy(), want)
    ctx.sync()
    t.free()


@pytest.mark.parametrize("bits", [8, 4])
def test_fused_fill_extreme_rows_match_fill(ctx, bits):
    """The GEMV's fused fill picks the same row scaling as the fill kernel:
    identical bits, RMSNorm of a huge row and a plain tiny row."""
    import torch
    from chpe_qwen35_hybrid_engine_b200 import X_F32, _lib as L
    rng = np.random.default_rng(3 + bits)
    N, K, M = 640, 4096, 2
    t, (codes, s, z, group) = _tensor(ctx, rng, bits, N, K)
    xf = ctx.xfrag(t, M, X_F32)
    x = torch.from_numpy(_rows(rng, M, K, [1e9, 1e-25])).cuda()
    gamma = torch.from_numpy((1 + 0.1 * rng.standard_normal(K)).astype(np.float32)).cuda()
    for op, aux in ((L.XOP_PLAIN, None), (L.XOP_RMSNORM, gamma)):
        ctx.xfrag_fill_op(xf, op, x, aux, eps=1e-6)
        ref = torch.empty(M, N, device="cuda")
        ctx.gemv_xfrag(t, xf, ref)
        got = torch.empty(M, N, device="cuda")
        ctx.gemv_src([t], [got], op, x, aux, M=M, eps=1e-6)
        torch.cuda.synchronize()
        assert torch.isfinite(got).all()
        assert torch.equal(got, ref), op
        if op == L.XOP_PLAIN:
            _check_rows(got.cpu().numpy(), O.gemv_grouped(codes, s, z, group, x.cpu().numpy(), num_workers=8))
    assert ctx.lib.chpe_sync(ctx.ptr) == 0
    xf.free()
    t.free()


@pytest.mark.parametrize("fmt", ["q8g32", "q4g64"])
@pytest.mark.parametrize("xdt", ["f32", "bf16"])
def test_prefill_extreme_rows(ctx, fmt, xdt):
    import torch
    rng = np.random.default_rng(11 + (fmt == "q4g64") + (2 if xdt == "bf16" else 0))
    M, N, K = 128, 384, 1024
    t, (codes, s, z, group) = _tensor(ctx, rng, 8 if fmt == "q8g32" else 4, N, K)
    x = _rows(rng, M, K, MAGS)
    xd = torch.from_numpy(x).cuda()
    if xdt == "bf16":
        xd = xd.to(torch.bfloat16)
    y = ctx.gemm_prefill(t, xd)
    torch.cuda.synchronize()
    ctx.sync()
    want = O.gemv_grouped(codes, s, z, group, xd.float().cpu().numpy(), num_workers=8)
    _check_rows(y.cpu().numpy(), want)
    t.free()
