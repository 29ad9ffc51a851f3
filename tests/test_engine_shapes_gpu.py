"""Greedy decode at the benchmark models' own widths against the oracle's
restatement of the reference step (src/engine.zig:583-1095).

* Qwen3.5-9B shape: hidden 4096, FFN 12288, GQA 16 q / 4 kv heads of 256,
  Gated-DeltaNet projections 6144 / 2048, vocab 151936 -- with 4 of the 32
  layers (3 Gated-DeltaNet + 1 full attention, the model's 3:1 pattern), so
  the oracle's fp64 CPU GEMVs finish in seconds per step.  64 greedy steps at
  batch 1 (w8a8 and q8g32), 16 verify steps at batch 4 and 8.
* Qwen2.5-72B shape: hidden 8192, FFN 29568, 64 q / 8 kv heads of 128, vocab
  152064, 4-bit codes with fp16 scale + zero per 64 -- 2 of the 80 layers,
  64 greedy steps.

Tokens must be identical at every step; the last step's logits within rel-L2
1e-3 (w8a8: the reference's integer arithmetic; the grouped formats: fp32
activations on fp32-accumulated tensor-core sums against fp64)."""
import dataclasses

import numpy as np
import pytest

from tests._util import rel_l2

pytestmark = pytest.mark.gpu


def _geom(which):
    from chpe_qwen35_hybrid_engine_b200.engine import QWEN25_72B, QWEN35_9B
    if which == "9b":
        return dataclasses.replace(QWEN35_9B, n_layers=4)
    return dataclasses.replace(QWEN25_72B, n_layers=2)


def _run(ctx, which, scheme, M, steps, seed):
    import torch
    from chpe_qwen35_hybrid_engine_b200.engine import build_random
    from oracle.engine_ref import EngineRef
    g = _geom(which)
    eng, host = build_random(ctx, g, scheme, seed=seed, keep_host=True, max_rows=8)
    ref = EngineRef(host, g, scheme)
    toks = [(1234 + 7 * i) % g.vocab for i in range(M)]
    got = eng.decode_greedy(toks, steps, M=M)
    want = ref.decode_greedy(toks, steps)
    assert np.array_equal(got, want), (np.nonzero((got != want).any(axis=1))[0][:5], got.ravel()[:16],
                                       want.ravel()[:16])
    last = [int(t) for t in want[-2]]
    _, logits = ref.step(last)
    eng.buf["tokens"][:M] = torch.tensor(last, dtype=torch.int32, device=eng.dev)
    eng.step(M)
    torch.cuda.synchronize()
    assert rel_l2(eng.buf["logits"][:M].cpu().numpy(), logits) < 1e-3
    eng.graphs.clear()


@pytest.mark.parametrize("scheme", ["w8a8", "q8g32"])
def test_9b_widths_greedy_64_steps(ctx, scheme):
    _run(ctx, "9b", scheme, 1, 64, seed=5)


@pytest.mark.parametrize("scheme", ["w8a8", "q8g32"])
@pytest.mark.parametrize("M", [4, 8])
def test_9b_widths_verify_16_steps(ctx, scheme, M):
    _run(ctx, "9b", scheme, M, 16, seed=6)


def test_72b_widths_q4g64_greedy_64_steps(ctx):
    _run(ctx, "72b", "q4g64", 1, 64, seed=9)
