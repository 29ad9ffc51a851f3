"""Tensor-parallel decode on 2 GPUs (NCCL) against the unsharded engine.

Both ranks draw the same full random-init weights and keep their shard
(column-split q/k/v/gate/up/LM head, row-split o/down).  The greedy tokens of
16 steps must equal those of the single-GPU engine on the same weights, and
the last step's logits must agree to fp32 summation-order noise (rel-L2 1e-5):
the only difference is that o and down partial sums meet in an all-reduce.
Needs 2 GPUs; skipped otherwise.
"""
import datetime
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _geom():
    from chpe_qwen35_hybrid_engine_b200.engine import Geometry
    # 2 GQA layers, 4 q heads / 2 kv heads of 128, hidden 512, FFN 1024, vocab 1000
    return Geometry(hidden=512, ffn=1024, vocab=1000, n_layers=2, attn_every=1, q_dim=512, kv_dim=256, ssm_qkv=0,
                    ssm_z=0, head_dim=128, q_heads=4, kv_heads=2)


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank(rank, world, port, scheme, q, allreduce="nccl"):
    import torch
    import torch.distributed as dist
    from chpe_qwen35_hybrid_engine_b200 import Context
    from chpe_qwen35_hybrid_engine_b200.tp import TensorParallelEngine
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        ctx = Context(rank)
        tp = TensorParallelEngine(ctx, _geom(), scheme, rank, world, seed=21, max_rows=8,
                                  allreduce="p2p" if allreduce.startswith("p2p") else allreduce)
        e = tp.eng
        e.fuse_exchange = allreduce != "p2p-separate"  # p2p: the all-reduce inside the next RMSNorm fill
        e.push_exchange = allreduce == "p2p-push"  # ... with the partials sent by the O / down GEMVs
        e.buf["tokens"][:1] = 33
        toks = []
        for _ in range(16):  # eager steps
            tp.step(1)
            toks.append(int(e.buf["argmax"][0]))
            e.buf["tokens"][:1] = e.buf["argmax"][:1]
        # the same 16 steps again, replaying a captured step
        g = tp.capture(1)
        gtoks = []
        e.buf["tokens"][:1] = 33
        for _ in range(16):
            g.replay()
            gtoks.append(int(e.buf["argmax"][0]))
            e.buf["tokens"][:1] = e.buf["argmax"][:1]
        torch.cuda.synchronize()
        # logits shard of the step from token 33
        e.buf["tokens"][:1] = 33
        tp.step(1)
        torch.cuda.synchronize()
        shard = e.buf["logits"][0, :e.head.rows].clone()
        parts = [torch.zeros(1000 // world, device=shard.device) for _ in range(world)]
        dist.all_gather(parts, shard)
        tp.graphs.clear()
        del g
        assert ctx.lib.chpe_sync(ctx.ptr) == 0  # no kernel recorded a timeout
        if rank == 0:
            q.put((toks, gtoks, torch.cat(parts).cpu().numpy()))
        dist.barrier()
        if tp.comm is not None:
            tp.comm.close()
        ctx.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("scheme,allreduce", [("q4g64", "p2p"), ("q4g64", "p2p-push"), ("q4g64", "p2p-separate"),
                                              ("q4g64", "nccl"), ("q8g32", "p2p")])
def test_tp2_decode_matches_single_gpu(ctx, scheme, allreduce):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from chpe_qwen35_hybrid_engine_b200.engine import build_random
    mpc = mp.get_context("spawn")
    q = mpc.Queue()
    port = _port()
    procs = [mpc.Process(target=_rank, args=(r, 2, port, scheme, q, allreduce)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        toks, gtoks, logits_tp = q.get(timeout=300)
    finally:
        for p in procs:
            p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs)
    eng, _ = build_random(ctx, _geom(), scheme, seed=21, max_rows=8)
    want = eng.decode_greedy([33], 16, M=1, use_graph=False)[:, 0].tolist()
    assert toks == want
    assert gtoks == want
    eng.buf["tokens"][:1] = 33
    eng.step(1)
    torch.cuda.synchronize()
    ref = eng.buf["logits"][0].cpu().numpy()
    assert np.linalg.norm(logits_tp - ref) / np.linalg.norm(ref) < 1e-5


def _fused_fill_check(ctx, comm, part, h0, rank):
    """chpe_allreduce_fill_dev against chpe_allreduce_residual_dev followed by
    the RMSNorm fill, on 8 rows of 8192 columns: hidden and the GEMV of the
    fragments must agree bit for bit (two exchanges each, both slot parities);
    then with the partial sent by a pushing GEMV (three exchanges each)."""
    import torch
    from chpe_qwen35_hybrid_engine_b200 import SCHEME_U_GROUP_F16_ZERO, X_F32, _lib as L
    from oracle import oracle as O
    from tests._util import pack_codes
    M, K, N = 8, 8192, 320
    rng = np.random.default_rng(77)  # the same weights on every rank
    codes, s, z = O.quantize_asym(rng.normal(0, 0.02, (N, K)).astype(np.float32), 4, 64)
    t = ctx.upload_matrix(4, SCHEME_U_GROUP_F16_ZERO, pack_codes(codes, 4), s, z, rows=N, cols=K, group=64)
    gamma = torch.from_numpy((1 + 0.1 * rng.standard_normal(K)).astype(np.float32)).cuda()
    xa, xb = ctx.xfrag(t, M, X_F32), ctx.xfrag(t, M, X_F32)
    p2 = part.view(M, K)
    ok = True
    for _ in range(2):
        ha = h0.view(M, K).cuda()
        hb = ha.clone()
        comm.allreduce_residual(p2, ha, M * K)
        ctx.xfrag_fill_op(xa, L.XOP_RMSNORM, ha, gamma, ldx=K, eps=1e-6)
        assert comm.allreduce_fill(p2, hb, xb, gamma, 1e-6)
        ya, yb = torch.empty(M, N, device="cuda"), torch.empty(M, N, device="cuda")
        ctx.gemv_xfrag(t, xa, ya)
        ctx.gemv_xfrag(t, xb, yb)
        torch.cuda.synchronize()
        ok = ok and torch.equal(ha, hb) and torch.equal(ya, yb)
    # the partial made by a pushing GEMV (chpe_gemv_xfrag_push_dev), collected
    # by the fill: the same bits as GEMV, all-reduce, fill
    Kin = 1024
    rr = np.random.default_rng(100 + rank)  # each rank its own projection
    c2, s2, z2 = O.quantize_asym(rr.normal(0, 0.02, (K, Kin)).astype(np.float32), 4, 64)
    t2 = ctx.upload_matrix(4, SCHEME_U_GROUP_F16_ZERO, pack_codes(c2, 4), s2, z2, rows=K, cols=Kin, group=64)
    xin = ctx.xfrag(t2, M, X_F32)
    for _ in range(3):
        ctx.xfrag_fill(xin, torch.from_numpy(rr.standard_normal((M, Kin)).astype(np.float32)).cuda())
        ha = h0.view(M, K).cuda()
        hc = ha.clone()
        pa, pc = torch.empty(M, K, device="cuda"), torch.empty(M, K, device="cuda")
        ctx.gemv_xfrag(t2, xin, pa)
        comm.allreduce_residual(pa, ha, M * K)
        ctx.xfrag_fill_op(xa, L.XOP_RMSNORM, ha, gamma, ldx=K, eps=1e-6)
        assert comm.gemv_push(t2, xin, pc)
        assert comm.allreduce_fill(pc, hc, xb, gamma, 1e-6, pushed=True)
        ya, yc = torch.empty(M, N, device="cuda"), torch.empty(M, N, device="cuda")
        ctx.gemv_xfrag(t, xa, ya)
        ctx.gemv_xfrag(t, xb, yc)
        torch.cuda.synchronize()
        ok = ok and torch.equal(pa, pc) and torch.equal(ha, hc) and torch.equal(ya, yc)
    xin.free()
    t2.free()
    xa.free()
    xb.free()
    t.free()
    return ok


def _comm_rank(rank, world, port, q, skip_rank):
    import torch
    import torch.distributed as dist
    from chpe_qwen35_hybrid_engine_b200 import Context
    from chpe_qwen35_hybrid_engine_b200.ops import Comm
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60))
    try:
        ctx = Context(rank)
        n = 8 * 8192
        comm = Comm(ctx, world, rank, n)
        comm.exchange()
        g = torch.Generator().manual_seed(5)
        parts = [torch.randn(n, generator=g) for _ in range(world)]
        h0 = torch.randn(n, generator=g)
        want = h0.clone()
        s = torch.zeros(n)
        for r in range(world):  # the kernel's order: sum of the partials in rank order, then add
            s = s + parts[r]
        want = h0 + s
        part = parts[rank].cuda()
        hidden = h0.cuda()
        refused = recovered = None
        merged = fused_same = None
        if skip_rank is None:
            for it in range(3):  # three epochs in a row (both slot parities)
                hidden.copy_(h0.cuda())
                comm.allreduce_residual(part, hidden, n)
                torch.cuda.synchronize()
            # the all-reduce fused into the RMSNorm fill: the same hidden bits and
            # the same fragments (seen through a GEMV) as all-reduce, then fill
            fused_same = _fused_fill_check(ctx, comm, part, h0, rank)
            # argmax merges interleaved with all-reduces (one sequence of epochs)
            merged = []
            for it in range(3):
                idx = torch.tensor(_MERGE_IDX[rank], dtype=torch.int32, device="cuda")
                val = torch.tensor(_MERGE_VAL[rank], dtype=torch.float32, device="cuda")
                comm.argmax_merge(idx, val, len(_MERGE_IDX[rank]), rank * 100)
                hidden.copy_(h0.cuda())
                comm.allreduce_residual(part, hidden, n)
                torch.cuda.synchronize()
                merged.append((idx.cpu().tolist(), val.cpu().tolist()))
            rc = ctx.lib.chpe_sync(ctx.ptr)
        else:
            if rank != skip_rank:
                comm.allreduce_residual(part, hidden, n)  # the peer never joins: the wait expires
                torch.cuda.synchronize()
            rc = ctx.lib.chpe_sync(ctx.ptr)
            if rank != skip_rank:
                # the failed object refuses the next exchange instead of pairing slots of different epochs
                from chpe_qwen35_hybrid_engine_b200._lib import ChpeError
                try:
                    comm.allreduce_residual(part, hidden, n)
                    refused = False
                except ChpeError as e:
                    refused = comm.failed() and e.code == -5
            # resynchronise every rank, then one exchange must be exact again
            comm.reset()
            hidden.copy_(h0.cuda())
            comm.allreduce_residual(part, hidden, n)
            torch.cuda.synchronize()
            recovered = ctx.lib.chpe_sync(ctx.ptr) == 0 and not comm.failed()
        out = (rank, rc, torch.equal(hidden.cpu(), want), refused, recovered, (merged, fused_same))
        dist.barrier()  # peers keep their receive areas mapped until everyone is done
        comm.close()
        ctx.close()
        q.put(out)
    finally:
        dist.destroy_process_group()


# Per-rank local argmax pairs of five rows (vocabulary shards of 100 rows):
# rank 1 wins; rank 0 wins; a tie won by rank 0's smaller global index (50 <
# 103); a tie won by rank 1's (103 < 150); negative values.
_MERGE_IDX = [[7, 9, 50, 150, 2], [3, 4, 3, 3, 8]]
_MERGE_VAL = [[1.0, 5.0, 2.5, 2.5, -3.0], [2.0, 4.0, 2.5, 2.5, -1.0]]


def _merge_want():
    from chpe_qwen35_hybrid_engine_b200.tp import merge_argmax
    out = []
    for m in range(5):
        vals = np.array([_MERGE_VAL[r][m] for r in (0, 1)], np.float32)
        idxs = np.array([_MERGE_IDX[r][m] + 100 * r for r in (0, 1)])
        out.append(merge_argmax(vals, idxs)[0])
    return out


@pytest.mark.parametrize("skip_rank", [None, 1])
def test_p2p_allreduce_exact_and_timeout(ctx, skip_rank):
    """The one-shot NVLink all-reduce: every rank's hidden state equals
    h0 + (sum of the partials in rank order) bit for bit, over three epochs.
    With skip_rank = 1 that rank never joins the first exchange: rank 0's
    bounded wait runs out (about 1 s), the kernel returns, chpe_sync reports
    CHPE_ETIMEOUT -- no GPU fault, the context stays usable -- and the comm
    object is marked failed, so rank 0's next exchange is refused rather than
    run with the ranks' epochs out of step.  After chpe_comm_reset on both
    ranks (between host barriers) an exchange is exact again."""
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    mpc = mp.get_context("spawn")
    q = mpc.Queue()
    port = _port()
    procs = [mpc.Process(target=_comm_rank, args=(r, 2, port, q, skip_rank)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    try:
        for _ in range(2):
            rank, rc, equal, refused, recovered, merged = q.get(timeout=120)
            res[rank] = (rc, equal, refused, recovered, merged)
    finally:
        for p in procs:
            p.join(timeout=60)
    assert all(p.exitcode == 0 for p in procs)
    if skip_rank is None:
        assert res[0][:2] == (0, True) and res[1][:2] == (0, True)
        # the argmax merge: identical global pairs on both ranks, every time
        want = (_merge_want(), [max(a, b) for a, b in zip(*_MERGE_VAL)])
        for r in (0, 1):
            for idx, val in res[r][4][0]:
                assert (idx, val) == want
            assert res[r][4][1] is True  # fused exchange + fill == all-reduce, then fill
    else:
        assert res[0][0] == -5  # CHPE_ETIMEOUT from rank 0's expired wait
        assert res[0][2] is True  # the failed object refused the next exchange
        assert res[0][3] and res[1][3]  # after the reset: exact on both ranks
        assert res[0][1] and res[1][1]

