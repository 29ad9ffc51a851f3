"""Token mixers on the GPU against the oracle's restatement (oracle/mixers_ref.py).

* GQA decode attention with RoPE and an fp32 KV cache (src/qwen72b_engine.zig:
  90-111, :291-369; src/chpe_engine.zig:191-212, :690-745): the 72B head
  layout (64 q / 8 kv heads of 128), the 9B layout (16 q / 4 kv heads of 256
  with the per-head output gate) and a small one; steps of 1, 3, 4 and 8
  rows at increasing positions, across the kernel's 64-position splits, up to
  a context of ~1100.  The rotated keys and values in the cache are the
  oracle's bit for bit (the same float32 operations; RoPE's pow / cos / sin
  in float64 on both sides); the attention outputs agree to float32
  summation order (rel-L2 <= 1e-5, far inside the path's 1e-3).
* Gated-DeltaNet conv1d + recurrence (src/ssm.zig:11-99): the 9B layout (16
  heads, key and value dim 128); steps of 1, 4, 8 and 2 rows from an empty
  state; outputs rel-L2 <= 1e-5, the state after every step bit for bit
  (conv and update are the same float32 operations in the same order).
"""
import numpy as np
import pytest

from oracle.mixers_ref import AttnLayerRef, DeltaLayerRef
from tests._util import rel_l2

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("qh,kvh,hd,gated,max_seq,plan", [
    (64, 8, 128, False, 1200, [1, 1, 8] + [8] * 130 + [3, 1, 4]),
    (16, 4, 256, True, 700, [1, 4] + [8] * 70 + [1, 8]),
    (4, 2, 64, False, 200, [1, 2, 3, 8, 8, 1] * 6),
])
def test_attention_against_oracle(ctx, qh, kvh, hd, gated, max_seq, plan):
    import torch
    rng = np.random.default_rng(qh + hd)
    theta = 1e6
    ldq = qh * hd * (2 if gated else 1)
    ref = AttnLayerRef(max_seq, qh, kvh, hd, theta, gated)
    kc = torch.zeros(max_seq, kvh, hd, device="cuda")
    vc = torch.zeros(max_seq, kvh, hd, device="cuda")
    pos = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = torch.empty(8, qh * hd, device="cuda")
    p = 0
    checked = 0
    for i, M in enumerate(plan):
        q = rng.standard_normal((M, ldq)).astype(np.float32)
        k = rng.standard_normal((M, kvh * hd)).astype(np.float32)
        v = rng.standard_normal((M, kvh * hd)).astype(np.float32)
        ctx.attn_decode(torch.from_numpy(q).cuda(), torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda(), kc, vc,
                        pos, M, qh, kvh, hd, theta, gated, out)
        ctx.pos_advance(pos, M)
        want = ref.step(q, k, v, p)
        p += M
        if i % 7 == 0 or i >= len(plan) - 3:  # the oracle is slow at long contexts: check a sample
            got = out[:M].cpu().numpy()
            assert np.isfinite(got).all()
            assert rel_l2(got, want) < 1e-5, (i, p, rel_l2(got, want))
            checked += 1
    torch.cuda.synchronize()
    assert int(pos.item()) == p
    assert np.array_equal(kc[:p].cpu().numpy(), ref.kc[:p])
    assert np.array_equal(vc[:p].cpu().numpy(), ref.vc[:p])
    assert ctx.lib.chpe_sync(ctx.ptr) == 0
    assert checked >= 3


def test_attention_refuses_a_full_cache(ctx):
    """A step past max_seq writes nothing and records an error (no fault)."""
    import torch
    qh, kvh, hd, max_seq = 4, 2, 64, 8
    kc = torch.zeros(max_seq, kvh, hd, device="cuda")
    vc = torch.zeros(max_seq, kvh, hd, device="cuda")
    pos = torch.tensor([6], dtype=torch.int32, device="cuda")
    q = torch.randn(4, qh * hd, device="cuda")
    kv = torch.randn(4, kvh * hd, device="cuda")
    out = torch.zeros(4, qh * hd, device="cuda")
    ctx.attn_decode(q, kv, kv, kc, vc, pos, 4, qh, kvh, hd, 1e6, False, out)
    torch.cuda.synchronize()
    assert ctx.lib.chpe_sync(ctx.ptr) == -1  # CHPE_EINVAL recorded, then cleared
    assert not kc.any() and not out.any()
    assert ctx.lib.chpe_sync(ctx.ptr) == 0


def test_deltanet_against_oracle(ctx):
    import torch
    rng = np.random.default_rng(3)
    H, dk, dv = 16, 128, 128
    C = H * (2 * dk + dv)
    conv_w = (rng.standard_normal((C, 4)) * 0.4).astype(np.float32)
    decay = rng.uniform(0.5, 0.95, H).astype(np.float32)
    ref = DeltaLayerRef(H, dk, dv, conv_w, decay)
    ring = torch.zeros(16, C, device="cuda")
    state = torch.zeros(H, dk, dv, device="cuda")
    pos = torch.zeros(1, dtype=torch.int32, device="cuda")
    out = torch.empty(8, H * dv, device="cuda")
    cw = torch.from_numpy(conv_w).cuda()
    dc = torch.from_numpy(decay).cuda()
    for M in (1, 4, 8, 2, 1, 8, 3):
        x = rng.standard_normal((M, C)).astype(np.float32)
        ctx.deltanet_step(torch.from_numpy(x).cuda(), cw, ring, state, dc, pos, M, H, dk, dv, out)
        ctx.pos_advance(pos, M)
        want = ref.step(x)
        got = out[:M].cpu().numpy()
        assert np.isfinite(got).all()
        assert rel_l2(got, want) < 1e-5, (M, rel_l2(got, want))
        assert np.array_equal(state.cpu().numpy(), ref.S)  # the same float32 operations, element by element
    assert ctx.lib.chpe_sync(ctx.ptr) == 0
