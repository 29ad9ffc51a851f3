"""Packed 4-bit and 2-bit GEMV at every shape of the benchmark sweep.

Weights are N(0, 0.02) quantized per 64 columns to unsigned codes with an
fp16 scale and zero (the library's device quantizer, bit-exact with the
oracle's restatement in tests/test_gemv_gpu.py), codes packed LSB first;
activations bf16 N(0, 1) at M = 1, 4 and 8; y fp32.  Shapes (K, N): (4096,
4096), (4096, 12288), (12288, 4096), (4096, 151936).  The reference is a torch
fp64 matmul with the dequantized weights (row blocks, on the device): bf16
activations reach the tensor cores exactly, so the only error is fp32
accumulation order -- bound 1e-4, well inside the path's 1e-3 (TOL)."""
import pytest

pytestmark = pytest.mark.gpu
TOL = 1e-3
SHAPES = [(4096, 4096), (4096, 12288), (12288, 4096), (4096, 151936)]


def _quantized(ctx, bits, K, N, seed):
    import torch
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    w = torch.empty(N, K, device="cuda")
    step = max(1, (1 << 26) // K)
    for r0 in range(0, N, step):
        w[r0:r0 + step].normal_(0.0, 0.02, generator=g)
    codes, s, z = ctx.quantize_group_dev(w, bits, 64, symmetric=False)
    del w
    per = 8 // bits
    packed = torch.zeros(N, K // per, dtype=torch.uint8, device="cuda")
    for j in range(per):
        packed |= codes[:, j::per] << (bits * j)
    return codes, packed.contiguous(), s, z


def _ref(codes, s, z, x):
    import torch
    N, K = codes.shape
    out = torch.empty(x.shape[0], N, dtype=torch.float64, device="cuda")
    xd = x.double()
    step = 16384
    for r0 in range(0, N, step):
        c = codes[r0:r0 + step].double()
        sc = s[r0:r0 + step].double().repeat_interleave(64, dim=1)
        zz = z[r0:r0 + step].double().repeat_interleave(64, dim=1)
        out[:, r0:r0 + step] = xd @ ((c - zz) * sc).T
    return out


@pytest.mark.parametrize("bits", [4, 2])
@pytest.mark.parametrize("K,N", SHAPES)
def test_config2_shapes(ctx, bits, K, N):
    import torch
    from chpe_qwen35_hybrid_engine_b200 import SCHEME_U_GROUP_F16_ZERO
    codes, packed, s, z = _quantized(ctx, bits, K, N, seed=bits * 10 + K + N)
    torch.cuda.synchronize()
    t = ctx.upload_matrix(bits, SCHEME_U_GROUP_F16_ZERO, packed, s, z, rows=N, cols=K, group=64)
    del packed
    g = torch.Generator(device="cuda")
    g.manual_seed(N)
    for M in (1, 4, 8):
        x = torch.randn(M, K, device="cuda", generator=g).to(torch.bfloat16)
        y = ctx.gemv(t, x)
        want = _ref(codes, s, z, x)
        torch.cuda.synchronize()
        assert torch.isfinite(y).all()
        err = (torch.linalg.norm(y.double() - want) / torch.linalg.norm(want)).item()
        assert err < TOL, (M, err)
        assert err < 1e-4, (M, err)
    assert ctx.lib.chpe_sync(ctx.ptr) == 0
    t.free()
