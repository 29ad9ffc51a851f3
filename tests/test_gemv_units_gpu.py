"""GPU tests of the GEMV work scheduling at full decode sizes.

The decode GEMV hands out its work as units drawn from per-slice atomic
counters (whole strip groups first, then chunks of blocks) and finishes
chunked strip groups by an acquire-release arrival count.  These tests cover
the shapes where every part of that runs -- several rounds of whole strip
groups, chunked tails, several K-slices, two and more rows -- against a torch
fp64 dequant-matmul, and check that results are bitwise identical from launch
to launch while launches of different shapes interleave (the counters reset
themselves at the end of every launch).
"""
import numpy as np
import pytest

from tests._util import rel_l2

pytestmark = pytest.mark.gpu
TOL = 1e-3  # rel-L2 bound of the path; fp32 activations land near 1e-6


def _q4(ctx, gen, N, K, group=64):
    import torch
    from chpe_qwen35_hybrid_engine_b200 import SCHEME_U_GROUP_F16_ZERO
    packed = torch.randint(0, 256, (N, K // 2), dtype=torch.uint8, device="cuda", generator=gen)
    s = (torch.rand(N, K // group, device="cuda", generator=gen) * 0.01 + 1e-3).half()
    z = torch.randint(0, 16, (N, K // group), device="cuda", generator=gen).half()
    t = ctx.upload_matrix(4, SCHEME_U_GROUP_F16_ZERO, packed, s, z, rows=N, cols=K, group=group)
    codes = torch.stack([packed & 15, packed >> 4], dim=2).reshape(N, K).double()
    w = (codes - z.double().repeat_interleave(group, 1)) * s.double().repeat_interleave(group, 1)
    return t, w


def _q8(ctx, gen, N, K):
    import torch
    from chpe_qwen35_hybrid_engine_b200 import SCHEME_I8_GROUP_F16
    codes = torch.randint(-127, 128, (N, K), dtype=torch.int8, device="cuda", generator=gen)
    s = (torch.rand(N, K // 32, device="cuda", generator=gen) * 1e-3 + 1e-4).half()
    t = ctx.upload_matrix(8, SCHEME_I8_GROUP_F16, codes, s, rows=N, cols=K, group=32)
    return t, codes.double() * s.double().repeat_interleave(32, 1)


# (bits, rows, cols, activation rows, activation dtype)
CASES = [
    (4, 29568, 8192, 1, "f32"),   # 72B gate: one round of whole strip groups, chunked tail
    (4, 8192, 29568, 1, "f32"),   # 72B down: four K-slices
    (4, 65536, 4096, 1, "bf16"),  # LM-head-like: several rounds of whole strip groups
    (8, 12288, 4096, 2, "f32"),   # config-0 format, two rows: chunks only
    (4, 29568, 8192, 4, "f32"),   # four rows: whole strip groups, second-kernel sums
    (4, 12288, 4096, 8, "f32"),   # eight rows, two K-slices
]


def test_drawn_units_full_size_and_interleaved_launches(ctx):
    import torch
    gen = torch.Generator(device="cuda")
    gen.manual_seed(1234)
    mats, xs, refs = [], [], []
    for bits, N, K, M, xdt in CASES:
        t, w = _q4(ctx, gen, N, K) if bits == 4 else _q8(ctx, gen, N, K)
        x = torch.randn(M, K, device="cuda", generator=gen)
        if xdt == "bf16":
            x = x.to(torch.bfloat16)
        refs.append((x.double() @ w.T).cpu().numpy())
        del w
        mats.append(t)
        xs.append(x)
    torch.cuda.empty_cache()
    first = [None] * len(CASES)
    for rep in range(3):
        for i, (t, x) in enumerate(zip(mats, xs)):
            y = ctx.gemv(t, x)
            if rep == 0:
                first[i] = y.clone()
                err = rel_l2(y.cpu().numpy(), refs[i])
                assert err < TOL, (CASES[i], err)
                assert err < 1e-5, (CASES[i], err)
            else:
                assert torch.equal(y, first[i]), (CASES[i], rep)
    ctx.sync()
    for t in mats:
        t.free()


def test_fused_gate_up_full_size_deterministic(ctx):
    """72B-shape gate/up SwiGLU (one launch over both matrices) against torch fp64, twice."""
    import torch
    gen = torch.Generator(device="cuda")
    gen.manual_seed(77)
    N, K = 29568, 8192
    tg, wg = _q4(ctx, gen, N, K)
    tu, wu = _q4(ctx, gen, N, K)
    x = torch.randn(1, K, device="cuda", generator=gen)
    g = x.double() @ wg.T
    u = x.double() @ wu.T
    del wg, wu
    ref = (g / (1.0 + torch.exp(-g)) * u).cpu().numpy()
    y1 = ctx.gemv_gateup_swiglu(tg, tu, x)
    y2 = ctx.gemv_gateup_swiglu(tg, tu, x)
    assert rel_l2(y1.cpu().numpy(), ref) < TOL
    assert torch.equal(y1, y2)
    ctx.sync()
    tg.free()
    tu.free()
