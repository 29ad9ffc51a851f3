"""The decode / verify step with the real token mixers -- GQA attention with
RoPE over an fp32 KV cache (src/qwen72b_engine.zig:291-369) and the
Gated-DeltaNet conv1d + recurrence (src/ssm.zig:11-99) -- against the oracle
engine with the same mixers (oracle/engine_ref.py, oracle/mixers_ref.py).

Greedy tokens must be identical at every step and the last step's logits
within rel-L2 1e-3; the grouped formats carry fp32 activations (the W8A8
scheme re-quantizes every mixer output to int8, where float32 summation-order
differences in the mixers turn into flipped codes, so it is not used here).
Rows of an M-row step are consecutive positions; a context is prefilled in
steps of 8 positions before decoding."""
import dataclasses

import numpy as np
import pytest

from tests._util import rel_l2

pytestmark = pytest.mark.gpu


def small_geom(**kw):
    from chpe_qwen35_hybrid_engine_b200.engine import Geometry
    # 4 layers (3 Gated-DeltaNet, 1 gated GQA: 4 q / 2 kv heads of 64), hidden 256,
    # DeltaNet 2 heads (key dim 128, value dim 64), vocab 1000
    g = Geometry(hidden=256, ffn=512, vocab=1000, n_layers=4, attn_every=4, q_dim=512, kv_dim=128, ssm_qkv=640,
                 ssm_z=128, q_heads=4, kv_heads=2, ssm_heads=2, mixer="real", max_seq=256)
    return dataclasses.replace(g, **kw)


def _compare(ctx, g, scheme, seed, context, steps, M):
    import torch
    from chpe_qwen35_hybrid_engine_b200.engine import build_random
    from oracle.engine_ref import EngineRef
    eng, host = build_random(ctx, g, scheme, seed=seed, keep_host=True, max_rows=8)
    ref = EngineRef(host, g, scheme)
    if len(context):
        eng.prefill(context, M=8)
        for i in range(0, len(context), 8):
            ref.step(list(context[i:i + 8]))
        assert int(eng.pos.item()) == ref.pos == len(context)
    toks = [(77 + 13 * i) % g.vocab for i in range(M)]
    got = eng.decode_greedy(toks, steps, M=M)
    want = ref.decode_greedy(toks, steps)
    assert np.array_equal(got, want), (np.nonzero((got != want).any(axis=1))[0][:5])
    assert int(eng.pos.item()) == ref.pos
    # one more step from the same tokens: logits agree
    last = [int(t) for t in want[-1]]
    _, logits = ref.step(last)
    eng.buf["tokens"][:M] = torch.tensor(last, dtype=torch.int32, device=eng.dev)
    eng.step(M)
    torch.cuda.synchronize()
    assert rel_l2(eng.buf["logits"][:M].cpu().numpy(), logits) < 1e-3
    assert ctx.lib.chpe_sync(ctx.ptr) == 0
    eng.graphs.clear()


@pytest.mark.parametrize("scheme", ["q8g32", "q4g64"])
def test_real_mixers_greedy_64_steps(ctx, scheme):
    _compare(ctx, small_geom(), scheme, seed=3, context=[], steps=64, M=1)


@pytest.mark.parametrize("M", [4, 8])
def test_real_mixers_verify_after_context(ctx, M):
    rng = np.random.default_rng(M)
    ctx_tokens = rng.integers(0, 1000, 43).astype(np.int32)  # 5 steps of 8 and a partial one
    _compare(ctx, small_geom(), "q8g32", seed=4, context=ctx_tokens, steps=12, M=M)


def test_real_mixers_9b_widths(ctx):
    from chpe_qwen35_hybrid_engine_b200.engine import QWEN35_9B
    g = dataclasses.replace(QWEN35_9B, n_layers=4, mixer="real", max_seq=512)
    rng = np.random.default_rng(9)
    _compare(ctx, g, "q8g32", seed=5, context=rng.integers(0, g.vocab, 64).astype(np.int32), steps=32, M=1)


def test_real_mixers_72b_widths(ctx):
    from chpe_qwen35_hybrid_engine_b200.engine import QWEN25_72B
    g = dataclasses.replace(QWEN25_72B, n_layers=2, mixer="real", max_seq=512)
    rng = np.random.default_rng(10)
    _compare(ctx, g, "q4g64", seed=6, context=rng.integers(0, g.vocab, 64).astype(np.int32), steps=32, M=1)
