"""Fused producers into activation fragments (chpe_xfrag_fill_op_dev) against
the unfused route: the producer's output computed on its own (the oracle's
rmsnorm / siluMul, the stand-in mixers restated in numpy), then the oracle's
grouped GEMV.  fp32 activations are split into fp16 hi + lo, so the bound is
far tighter than the path's 1e-3: 1e-4, because for 2-bit codes read at bit 6
the activations are pre-scaled by 2^-6 and the lo half of a small one falls
into fp16's subnormal range (absolute step 2^-24).

TIGHT below is that bound."""
import numpy as np
import pytest

from oracle import oracle as O
from tests._util import pack_codes, rel_l2

pytestmark = pytest.mark.gpu
TIGHT = 1e-4


def _silu(v):
    return v / (1.0 + np.exp(-v))


def _tensor(ctx, rng, bits, N, K):
    from chpe_qwen35_hybrid_engine_b200 import SCHEME_I8_GROUP_F16, SCHEME_U_GROUP_F16_ZERO
    w = rng.normal(0, 0.02, (N, K)).astype(np.float32)
    if bits == 8:
        codes, s = O.quantize_sym8(w, 32)
        t = ctx.upload_matrix(8, SCHEME_I8_GROUP_F16, codes, s, rows=N, cols=K, group=32)
        return t, lambda x: O.gemv_grouped(codes, s, None, 32, x, num_workers=8)
    codes, s, z = O.quantize_asym(w, bits, 64)
    t = ctx.upload_matrix(bits, SCHEME_U_GROUP_F16_ZERO, pack_codes(codes, bits), s, z, rows=N, cols=K, group=64)
    return t, lambda x: O.gemv_grouped(codes, s, z, 64, x, num_workers=8)


@pytest.mark.parametrize("bits", [8, 4, 2])
@pytest.mark.parametrize("M", [1, 3, 8])
def test_fill_ops_match_unfused(ctx, bits, M):
    import torch
    from chpe_qwen35_hybrid_engine_b200 import X_F32, _lib as L
    rng = np.random.default_rng(bits * 10 + M)
    N, K = 384, 2048
    t, ref_gemv = _tensor(ctx, rng, bits, N, K)
    xf = ctx.xfrag(t, M, X_F32)
    y = torch.empty(M, N, device="cuda")

    def run():
        ctx.gemv_xfrag(t, xf, y)
        torch.cuda.synchronize()
        return y.cpu().numpy()

    # RMSNorm (x rows with a stride wider than K)
    x = (rng.standard_normal((M, K + 64)) * 3).astype(np.float32)
    gamma = (1 + 0.1 * rng.standard_normal(K)).astype(np.float32)
    ctx.xfrag_fill_op(xf, L.XOP_RMSNORM, torch.from_numpy(x).cuda(), torch.from_numpy(gamma).cuda(), ldx=K + 64,
                      eps=1e-6)
    xn = np.stack([O.rmsnorm(r[:K], gamma, 1e-6) for r in x])
    assert rel_l2(run(), ref_gemv(xn)) < TIGHT
    # SiLU * mul
    g_ = rng.standard_normal((M, K)).astype(np.float32)
    u_ = rng.standard_normal((M, K)).astype(np.float32)
    ctx.xfrag_fill_op(xf, L.XOP_SILU_MUL, torch.from_numpy(g_).cuda(), torch.from_numpy(u_).cuda())
    assert rel_l2(run(), ref_gemv(np.stack([O.silu_mul(a, b) for a, b in zip(g_, u_)]))) < TIGHT
    # attention stand-in, reference form (out[i] = v[i % kv]) and head-aligned GQA form
    kv = 512
    v = rng.standard_normal((M, kv)).astype(np.float32)
    ctx.xfrag_fill_op(xf, L.XOP_ATTN_STUB, torch.from_numpy(v).cuda(), ldx=kv, kv_dim=kv)
    assert rel_l2(run(), ref_gemv(v[:, np.arange(K) % kv])) < TIGHT
    hd, grp = 128, 4
    ctx.xfrag_fill_op(xf, L.XOP_ATTN_STUB, torch.from_numpy(v).cuda(), ldx=kv, kv_dim=kv, head_dim=hd, group=grp)
    src = ((np.arange(K) // hd) // grp) * hd + np.arange(K) % hd
    assert rel_l2(run(), ref_gemv(v[:, src])) < TIGHT
    # Gated-DeltaNet stand-in, both forms
    qd = 768
    q = rng.standard_normal((M, qd)).astype(np.float32)
    z = rng.standard_normal((M, K)).astype(np.float32)
    for son in (False, True):
        ctx.xfrag_fill_op(xf, L.XOP_SSM_STUB, torch.from_numpy(q).cuda(), torch.from_numpy(z).cuda(), ldx=qd,
                          qkv_dim=qd, silu_on_qkv=son)
        qq = q[:, np.arange(K) % qd]
        want = _silu(qq) * z if son else qq * _silu(z)
        assert rel_l2(run(), ref_gemv(want.astype(np.float32))) < TIGHT
    # plain fill through the op entry point equals chpe_xfrag_fill_dev bit for bit
    xp = torch.from_numpy(rng.standard_normal((M, K)).astype(np.float32)).cuda()
    ctx.xfrag_fill_op(xf, L.XOP_PLAIN, xp)
    a = run()
    ctx.xfrag_fill(xf, xp)
    assert np.array_equal(a, run())
    xf.free()
    t.free()


def test_fill_op_errors(ctx):
    import torch
    from chpe_qwen35_hybrid_engine_b200 import ChpeError, X_BF16, X_F32, _lib as L
    rng = np.random.default_rng(1)
    t, _ = _tensor(ctx, rng, 4, 64, 256)
    xf = ctx.xfrag(t, 1, X_BF16)
    x = torch.zeros(1, 256, device="cuda")
    with pytest.raises(ChpeError):  # fused producers need fp32 fragments
        ctx.xfrag_fill_op(xf, L.XOP_RMSNORM, x, x[0])
    with pytest.raises(ChpeError):  # dtype mismatch
        ctx.xfrag_fill_op(xf, L.XOP_PLAIN, x, x_dtype=X_F32)
    xf.free()
    xf = ctx.xfrag(t, 1, X_F32)
    with pytest.raises(ChpeError):  # rmsnorm without gamma
        ctx.xfrag_fill_op(xf, L.XOP_RMSNORM, x)
    with pytest.raises(ChpeError):  # unknown op
        ctx.xfrag_fill_op(xf, 99, x)
    xf.free()
    t.free()


@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("M", [1, 3, 8])
def test_fused_fill_gemv_equals_fill_then_gemv(ctx, bits, M):
    """chpe_gemv_src_dev (each GEMV CTA builds its fragments from the source op,
    RMSNorm statistics included) gives the same bits as chpe_xfrag_fill_op_dev
    followed by the fragment GEMVs: plain, accumulate, three tensors in one
    launch, and gate/up SwiGLU.  Above two activation rows the fragment GEMV
    streams its activations through the weight ring in one K slice while the
    fused GEMV keeps them resident (split K), so the two sum the same products
    in different orders: there the bar is fp32 reordering, 2e-6 of the row
    maximum."""
    import torch
    from chpe_qwen35_hybrid_engine_b200 import X_F32, _lib as L
    rng = np.random.default_rng(100 + bits * 10 + M)
    K = 4096
    t0, _ = _tensor(ctx, rng, bits, 520, K)
    t1, _ = _tensor(ctx, rng, bits, 100, K)
    t2, _ = _tensor(ctx, rng, bits, 520, K)
    xf = ctx.xfrag(t0, M, X_F32)
    dev = "cuda"
    x = torch.from_numpy((rng.standard_normal((M, K + 32)) * 2).astype(np.float32)).to(dev)
    gamma = torch.from_numpy((1 + 0.1 * rng.standard_normal(K)).astype(np.float32)).to(dev)
    u = torch.from_numpy(rng.standard_normal((M, K)).astype(np.float32)).to(dev)
    v = torch.from_numpy(rng.standard_normal((M, 1024)).astype(np.float32)).to(dev)
    cases = [dict(op=L.XOP_RMSNORM, x=x, aux=gamma, ldx=K + 32, eps=1e-6),
             dict(op=L.XOP_SILU_MUL, x=x, aux=u, ldx=K + 32, ld_aux=K),
             dict(op=L.XOP_ATTN_STUB, x=v, ldx=1024, kv_dim=1024, head_dim=128, group=4),
             dict(op=L.XOP_SSM_STUB, x=v, aux=u, ldx=1024, ld_aux=K, qkv_dim=768, silu_on_qkv=M > 1),
             dict(op=L.XOP_PLAIN, x=x[:, :K].contiguous())]
    for kw in cases:
        ctx.xfrag_fill_op(xf, kw["op"], kw["x"], kw.get("aux"), ldx=kw.get("ldx", 0), ld_aux=kw.get("ld_aux", 0),
                          eps=kw.get("eps", 0.0), kv_dim=kw.get("kv_dim", 1), head_dim=kw.get("head_dim", 0),
                          group=kw.get("group", 1), qkv_dim=kw.get("qkv_dim", 1),
                          silu_on_qkv=kw.get("silu_on_qkv", False))
        ref = [torch.empty(M, t.rows, device=dev) for t in (t0, t1)]
        ctx.gemv_multi_xfrag([t0, t1], xf, ref)
        ref_gu = torch.empty(M, 520, device=dev)
        ctx.gemv_gateup_swiglu_xfrag(t0, t2, xf, ref_gu)
        base = torch.from_numpy(rng.standard_normal((M, 520)).astype(np.float32)).to(dev)
        ref_acc = base.clone()
        ctx.gemv_xfrag(t0, xf, ref_acc, accumulate=True)
        op = kw.pop("op")
        xx = kw.pop("x")
        aux = kw.pop("aux", None)
        got = [torch.empty(M, t.rows, device=dev) for t in (t0, t1)]
        ctx.gemv_src([t0, t1], got, op, xx, aux, M=M, **kw)
        got_gu = torch.empty(M, 520, device=dev)
        ctx.gemv_src([t0, t2], [got_gu], op, xx, aux, M=M, mode=1, **kw)
        got_acc = base.clone()
        ctx.gemv_src([t0], [got_acc], op, xx, aux, M=M, accumulate=True, **kw)
        torch.cuda.synchronize()

        def same(a, b):
            if M <= 2:
                return torch.equal(a, b)
            tol = 2e-6 * b.abs().amax(dim=1, keepdim=True)
            return bool(((a - b).abs() <= tol).all())
        assert same(got[0], ref[0]) and same(got[1], ref[1]), op
        assert same(got_gu, ref_gu), op
        assert same(got_acc, ref_acc), op
    assert ctx.lib.chpe_sync(ctx.ptr) == 0
    xf.free()
    for t in (t0, t1, t2):
        t.free()

