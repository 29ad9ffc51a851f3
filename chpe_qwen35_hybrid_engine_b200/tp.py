"""Tensor parallelism for the 72B-shape model: one process per GPU.

Partition (one exchange per block, as the model's structure allows):
  * q, k, v: column split by whole heads (64 q / 8 kv heads of 128 divide by
    2, 4, 8); the head-aligned attention stand-in then stays rank-local;
  * gate, up: column split on 64-column group boundaries, identical to the
    down projection's K split, so SwiGLU stays rank-local;
  * o, down: row (K) split on group boundaries (down's 462 groups split
    unevenly at 4 and 8 ranks: 115/116 and 57/58 groups);
  * after o and after down, the [M, hidden] fp32 partial sums are summed over
    the ranks and added to the replicated hidden state: by the library's
    one-shot NVLink all-reduce kernel (every rank pushes its partial into every
    peer's memory, then sums in rank order), or by NCCL;
  * the LM head is column split over the vocabulary; each rank takes its local
    argmax and the (value, index) pairs are exchanged and merged, ties to the
    smaller index as in src/engine.zig:1098-1110: by the library's P2P merge
    kernel with the one-shot all-reduce, or by NCCL all-gathers.
"""
from __future__ import annotations

import numpy as np

from .engine import Geometry, HybridEngine, build_random, build_random_codes


def shard_bounds(total: int, world: int, rank: int, group: int = 1) -> tuple[int, int]:
    """[start, end) of rank's contiguous share of `total` columns, on `group` boundaries."""
    ng = total // group
    return (rank * ng // world) * group, ((rank + 1) * ng // world) * group


def merge_argmax(values: np.ndarray, indices: np.ndarray) -> tuple[int, float]:
    """Global argmax from per-rank (max value, global index) pairs: the largest
    value wins, ties go to the smaller index."""
    best = 0
    for r in range(1, len(values)):
        if values[r] > values[best] or (values[r] == values[best] and indices[r] < indices[best]):
            best = r
    return int(indices[best]), float(values[best])


def merge_gathered(values, indices):
    """Row-wise global argmax from gathered per-rank pairs (torch tensors
    [world, M]): the largest value wins, ties go to the smaller index.
    Returns (indices [M] int32, values [M])."""
    import torch
    best_v = values.max(dim=0).values
    cand = torch.where(values == best_v[None, :], indices, torch.full_like(indices, 2 ** 31 - 1))
    return cand.min(dim=0).values.to(torch.int32), best_v


def partition(geom: Geometry, world: int, rank: int, group: int) -> dict:
    """Rows (output columns) and K ranges each projection has on `rank`:
    name -> (row_start, row_end, k_start, k_end) of the full matrix."""
    H, F = geom.hidden, geom.ffn
    part = {}
    col = lambda n: (rank * n // world, (rank + 1) * n // world)
    fr = shard_bounds(F, world, rank, group)
    if geom.head_dim:
        for name, n in (("q", geom.q_dim), ("k", geom.kv_dim), ("v", geom.kv_dim)):
            part[name] = col(n) + (0, H)
        part["o"] = (0, H) + shard_bounds(H, world, rank, group)
    part["gate"] = fr + (0, H)
    part["up"] = fr + (0, H)
    part["down"] = (0, H) + fr
    part["head"] = col(geom.vocab) + (0, H)
    return part


class TensorParallelEngine:
    def __init__(self, ctx, geom: Geometry, scheme: str, rank: int, world: int, seed: int = 0, max_rows: int = 8,
                 process_group=None, random_codes: bool = False, allreduce: str = "p2p"):
        """allreduce: "p2p" -- the library's one-shot NVLink all-reduce kernel
        (adds into the hidden state as well); "nccl" -- torch.distributed."""
        import torch
        import torch.distributed as dist
        self.rank, self.world, self.geom = rank, world, geom
        self.pg = process_group
        if random_codes:
            self.eng = build_random_codes(ctx, geom, scheme, seed=seed, max_rows=max_rows, shard=(rank, world))
        else:
            self.eng, _ = build_random(ctx, geom, scheme, seed=seed, max_rows=max_rows, shard=(rank, world))
        self.comm = None
        if world > 1 and allreduce == "p2p":
            from .ops import Comm
            self.comm = Comm(ctx, world, rank, max_rows * geom.hidden)
            self.comm.exchange(self.pg)
            self.eng.comm = self.comm
        elif world > 1:
            self.eng.allreduce = lambda t: dist.all_reduce(t, group=self.pg)
        self.v0 = rank * geom.vocab // world  # first vocabulary row of this rank's LM-head shard
        dev = self.eng.dev
        self.gather_v = torch.zeros(world, max_rows, dtype=torch.float32, device=dev)
        self.gather_i = torch.zeros(world, max_rows, dtype=torch.int32, device=dev)
        self.graphs = {}

    def step(self, M: int, stream=None):
        import torch
        import torch.distributed as dist
        e = self.eng
        e.step(M, stream)
        if self.world == 1:
            return
        if self.comm is not None:  # the library's exchange: one kernel, every rank gets the global pair
            self.comm.argmax_merge(e.buf["argmax"], e.buf["maxv"], M, self.v0, stream)
            return
        # NCCL: local argmax -> global index; all-gather the (value, index) pairs of every rank
        loc_i = (e.buf["argmax"][:M] + self.v0).to(torch.int32)
        loc_v = e.buf["maxv"][:M].clone()
        gv = [self.gather_v[r, :M] for r in range(self.world)]
        gi = [self.gather_i[r, :M] for r in range(self.world)]
        dist.all_gather(gv, loc_v, group=self.pg)
        dist.all_gather(gi, loc_i, group=self.pg)
        idx, val = merge_gathered(self.gather_v[:, :M], self.gather_i[:, :M])
        e.buf["argmax"][:M] = idx
        e.buf["maxv"][:M] = val

    def capture(self, M: int):
        import torch
        snap = self.eng._snapshot()
        st = torch.cuda.Stream(self.eng.dev)
        st.wait_stream(torch.cuda.current_stream(self.eng.dev))
        with torch.cuda.stream(st):
            self.step(M, st)
        torch.cuda.synchronize(self.eng.dev)
        self.eng._restore(snap)
        torch.cuda.synchronize(self.eng.dev)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=st):
            self.step(M, st)
        self.graphs[M] = g
        return g

    def reset(self):
        self.eng.reset()

    def prefill(self, tokens, M: int = 8):
        """Feed a context M positions at a time through the tensor-parallel step
        (every rank runs the same steps; a last partial chunk runs eagerly)."""
        import torch
        b = self.eng.buf
        toks = np.asarray(tokens, np.int32)
        if M not in self.graphs:
            self.capture(M)
        i = 0
        while i < len(toks):
            n = min(M, len(toks) - i)
            b["tokens"][:n].copy_(torch.from_numpy(toks[i:i + n]).to(self.eng.dev))
            if n == M:
                self.graphs[M].replay()
            else:
                self.step(n)
            i += n
        torch.cuda.synchronize(self.eng.dev)
