"""Prefill dequant-GEMM (tcgen05, M >= 64) against the oracle and torch fp64.

The weights are dequantized to fp16 (one rounding of q*s or (c-z)*s); each
activation row is scaled by a power of two into fp16's range, where bf16 and
fp16 values are exact and fp32 values take one rounding, so the result is
within ~2^-12 relative per term of the exact product: rel-L2 well under the
path's 1e-3 (TOL).  fp32 inputs are compared with the fp32 oracle itself.  Small
shapes are checked against the oracle's grouped GEMV (fp64 accumulation); the
full config-3 shapes (M = 2048) against a torch fp64 dequant-matmul.
"""
import numpy as np
import pytest

from oracle import oracle as O
from tests._util import pack_codes, rel_l2

pytestmark = pytest.mark.gpu
TOL = 1e-3


def _q8(ctx, rng, N, K):
    from chpe_qwen35_hybrid_engine_b200 import SCHEME_I8_GROUP_F16
    w = rng.normal(0, 0.02, (N, K)).astype(np.float32)
    codes, s = O.quantize_sym8(w, 32)
    t = ctx.upload_matrix(8, SCHEME_I8_GROUP_F16, codes, s, rows=N, cols=K, group=32)
    return t, (codes, s, None, 32)


def _q4(ctx, rng, N, K, group=64):
    from chpe_qwen35_hybrid_engine_b200 import SCHEME_U_GROUP_F16_ZERO
    w = rng.normal(0, 0.02, (N, K)).astype(np.float32)
    codes, s, z = O.quantize_asym(w, 4, group)
    t = ctx.upload_matrix(4, SCHEME_U_GROUP_F16_ZERO, pack_codes(codes, 4), s, z, rows=N, cols=K, group=group)
    return t, (codes, s, z, group)


def _dequant_torch(ref, dev):
    import torch
    codes, s, z, group = ref
    c = torch.from_numpy(codes.astype(np.float64)).to(dev)
    sc = torch.from_numpy(s.astype(np.float64)).to(dev).repeat_interleave(group, dim=1)
    if z is None:
        return c * sc
    zz = torch.from_numpy(z.astype(np.float64)).to(dev).repeat_interleave(group, dim=1)
    return (c - zz) * sc


@pytest.mark.parametrize("fmt", ["q8g32", "q4g64", "q4g128"])
@pytest.mark.parametrize("M,N,K,xdt", [(128, 256, 256, "bf16"), (200, 300, 320, "f32"), (64, 520, 1024, "bf16"),
                                       (384, 256, 2048, "f16")])
def test_prefill_small_against_oracle(ctx, fmt, M, N, K, xdt):
    import torch
    if fmt == "q4g128" and K % 128:
        pytest.skip("K not a multiple of the group")
    rng = np.random.default_rng(M + N + K)
    t, ref = _q8(ctx, rng, N, K) if fmt == "q8g32" else _q4(ctx, rng, N, K, 64 if fmt == "q4g64" else 128)
    x32 = rng.standard_normal((M, K)).astype(np.float32)
    dt = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}[xdt]
    xd = torch.from_numpy(x32).cuda().to(dt)
    y = ctx.gemm_prefill(t, xd)
    torch.cuda.synchronize()
    ctx.sync()
    xo = xd.float().cpu().numpy()
    codes, s, z, group = ref
    want = O.gemv_grouped(codes, s, z, group, xo, num_workers=8)
    got = y.cpu().numpy()
    assert np.isfinite(got).all()
    # fp32 activations are compared with the fp32 oracle: the kernel scales each
    # row by a power of two and rounds it to fp16 once (~2^-12 relative per value)
    assert rel_l2(got, want) < TOL, rel_l2(got, want)
    assert rel_l2(got, want) < (5e-4 if xdt == "f32" else 3e-4)
    # accumulate into an existing y, and determinism
    y0 = torch.from_numpy(rng.standard_normal((M, N)).astype(np.float32)).cuda()
    y1 = y0.clone()
    ctx.gemm_prefill(t, xd, out=y1, accumulate=True)
    assert rel_l2(y1.cpu().numpy(), y0.cpu().numpy() + got) < 1e-6
    assert torch.equal(ctx.gemm_prefill(t, xd), y)
    t.free()


@pytest.mark.parametrize("fmt", ["q8g32", "q4g64"])
@pytest.mark.parametrize("K,N", [(4096, 12288), (12288, 4096), (4096, 6144)])
def test_prefill_config3_full_size(ctx, fmt, K, N):
    """M = 2048 bf16 activations N(0,1) against torch fp64 on the dequantized weights."""
    import torch
    rng = np.random.default_rng(K + N)
    t, ref = _q8(ctx, rng, N, K) if fmt == "q8g32" else _q4(ctx, rng, N, K)
    M = 2048
    xd = torch.from_numpy(rng.standard_normal((M, K)).astype(np.float32)).cuda().to(torch.bfloat16)
    y = ctx.gemm_prefill(t, xd)
    ctx.sync()
    wd = _dequant_torch(ref, xd.device)
    want = xd.double() @ wd.T
    del wd
    err = (torch.linalg.norm(y.double() - want) / torch.linalg.norm(want)).item()
    assert err < TOL, err
    assert err < 3e-4, err
    t.free()


def test_prefill_unsupported_format(ctx):
    import torch
    from chpe_qwen35_hybrid_engine_b200 import ChpeError, SCHEME_U_GROUP_F16_ZERO
    rng = np.random.default_rng(3)
    w = rng.normal(0, 0.02, (64, 256)).astype(np.float32)
    codes, s, z = O.quantize_asym(w, 2, 64)
    t = ctx.upload_matrix(2, SCHEME_U_GROUP_F16_ZERO, pack_codes(codes, 2), s, z, rows=64, cols=256, group=64)
    with pytest.raises(ChpeError):
        ctx.gemm_prefill(t, torch.zeros(128, 256, device="cuda", dtype=torch.bfloat16))
    t.free()
