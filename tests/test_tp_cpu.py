"""Tensor-parallel partition of the 72B-shape model, checked on the CPU.

Two `gloo` ranks (127.0.0.1) stand in for two GPUs: each computes its shard's
partial GEMV with the oracle, the partials are summed with an all-reduce and
must equal the unsharded GEMV; the vocabulary-split argmax, gathered and
merged, must equal the global argmax (ties to the smaller index, as
src/engine.zig:1098-1110).  The partition itself is checked at 2, 4 and 8
ranks: head-aligned q/k/v, group-aligned K splits that tile every row
exactly once, gate/up rows equal to down's K range.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from chpe_qwen35_hybrid_engine_b200.engine import QWEN25_72B, _row_split
from chpe_qwen35_hybrid_engine_b200.tp import merge_argmax, merge_gathered, partition, shard_bounds


@pytest.mark.parametrize("world", [2, 4, 8])
def test_partition_covers_each_weight_once(world):
    g = QWEN25_72B
    parts = [partition(g, world, r, 64) for r in range(world)]
    full = {"q": (g.q_dim, g.hidden), "k": (g.kv_dim, g.hidden), "v": (g.kv_dim, g.hidden), "o": (g.hidden, g.hidden),
            "gate": (g.ffn, g.hidden), "up": (g.ffn, g.hidden), "down": (g.hidden, g.ffn),
            "head": (g.vocab, g.hidden)}
    for name, (R, K) in full.items():
        total = 0
        for p in parts:
            r0, r1, k0, k1 = p[name]
            assert 0 <= r0 <= r1 <= R and 0 <= k0 <= k1 <= K
            assert k0 % 64 == 0 and k1 % 64 == 0 or (k0, k1) == (0, K)
            total += (r1 - r0) * (k1 - k0)
        assert total == R * K, name
    for r, p in enumerate(parts):
        # q / k / v split on whole heads
        for name in ("q", "k", "v"):
            r0, r1, _, _ = p[name]
            assert r0 % g.head_dim == 0 and r1 % g.head_dim == 0
        # q heads of this rank map onto its own kv heads (GQA group stays local)
        q_heads = (p["q"][1] - p["q"][0]) // g.head_dim
        kv_heads = (p["k"][1] - p["k"][0]) // g.head_dim
        assert q_heads == kv_heads * (g.q_heads // g.kv_heads)
        # SwiGLU is rank-local: gate / up rows are exactly down's K range
        assert p["gate"][:2] == p["down"][2:] == p["up"][:2]
        # o's K range is this rank's attention output (its own q heads)
        assert p["o"][2:] == p["q"][:2]
        sl = _row_split(g.ffn, world, r, "q4g64")
        assert (sl.start, sl.stop) == p["down"][2:]


def test_shard_bounds_examples():
    assert shard_bounds(29568, 8, 3, 64) == (11072, 14784)
    assert shard_bounds(29568, 2, 1, 64) == (14784, 29568)
    assert shard_bounds(152064, 8, 7, 1) == (133056, 152064)
    assert merge_argmax(np.array([1.0, 3.0, 3.0]), np.array([5, 9, 2])) == (2, 3.0)


def test_merge_gathered_ties_and_rows():
    V = torch.tensor([[1.0, 5.0, 2.0], [3.0, 5.0, 2.0], [3.0, 4.0, 2.0]])
    I = torch.tensor([[10, 20, 30], [40, 7, 31], [2, 1, 29]], dtype=torch.int32)
    idx, val = merge_gathered(V, I)
    assert idx.tolist() == [2, 7, 29]
    assert val.tolist() == [3.0, 5.0, 2.0]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank_main(rank, world, port, out):
    from oracle import oracle as O
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(5)
        N, K, V = 96, 1024, 500
        codes = rng.integers(0, 16, (N, K), dtype=np.uint8)
        scales = (0.004 * np.exp(rng.normal(0, 0.25, (N, K // 64)))).astype(np.float16)
        zeros = rng.integers(6, 10, (N, K // 64)).astype(np.float16)
        x = rng.standard_normal((2, K)).astype(np.float32)
        k0, k1 = shard_bounds(K, world, rank, 64)
        g0, g1 = k0 // 64, k1 // 64
        part = O.gemv_grouped(np.ascontiguousarray(codes[:, k0:k1]), np.ascontiguousarray(scales[:, g0:g1]),
                              np.ascontiguousarray(zeros[:, g0:g1]), 64, np.ascontiguousarray(x[:, k0:k1]),
                              num_workers=1)
        t = torch.from_numpy(part.astype(np.float64))
        dist.all_reduce(t)
        full = O.gemv_grouped(codes, scales, zeros, 64, x, num_workers=1)
        err = float(np.abs(t.numpy() - full).max() / np.abs(full).max())
        # vocabulary-split argmax with a planted tie across the shard boundary
        logits = rng.standard_normal((2, V)).astype(np.float32)
        v0, v1 = rank * V // world, (rank + 1) * V // world
        logits[0, V // world - 1] = logits[0, V // world] = 50.0  # equal maxima on both sides of rank 0/1 boundary
        loc = logits[:, v0:v1]
        li = torch.from_numpy(loc.argmax(axis=1).astype(np.int32) + v0)
        lv = torch.from_numpy(loc.max(axis=1))
        gv = [torch.zeros_like(lv) for _ in range(world)]
        gi = [torch.zeros_like(li) for _ in range(world)]
        dist.all_gather(gv, lv)
        dist.all_gather(gi, li)
        idx, _ = merge_gathered(torch.stack(gv), torch.stack(gi))
        want = [O.argmax(r)[0] for r in logits]
        if rank == 0:
            out.put((err, idx.tolist(), want))
    finally:
        dist.destroy_process_group()


def test_two_rank_gloo_partial_sums_and_argmax():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        err, got, want = q.get(timeout=120)
    finally:
        for p in procs:
            p.join(timeout=60)
    assert all(p.exitcode == 0 for p in procs)
    assert err < 1e-6  # each partial is rounded to fp32 once
    assert got == want
    assert got[0] == 500 // 2 - 1  # the tie goes to the smaller index
