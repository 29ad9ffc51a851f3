"""Decode / speculative-verify step of the CHPE hybrid model on the B200 library.

Mirrors the reference's orchestration (src/engine.zig Qwen35Engine):
  step        (batch 1, :583-734)   fused gate/up SwiGLU, SSM stand-in qkv*silu(z)
  stepBatch4  (:753-900)            unfused gate, up + siluMul, SSM stand-in silu(qkv)*z
  stepBatch8  (:902-1095)           same as batch 4 with 8 rows
with the reference's stand-ins for the token mixers (full attention = V
broadcast, :619-623; Gated DeltaNet = qkv gated by z, :651-654) -- or, with
Geometry.mixer = "real", GQA attention with RoPE over an fp32 KV cache
(src/qwen72b_engine.zig:291-369) and the Gated-DeltaNet conv1d + recurrence
(src/ssm.zig:11-99), the output gated by silu(z) -- RMSNorm before each
block, residual adds, final RMSNorm, LM head and argmax (:1098-1110).  With
real mixers the rows of an M-row step are consecutive positions of one
sequence (speculative verification), and the position lives on the device.
Every projection runs on the library's quantized GEMV; the residual add is the
GEMV's accumulate into the hidden state.  A step of fixed row count is captured
once into a CUDA graph and replayed; greedy decoding feeds the argmax of one
step into the next without leaving the device.

Weight schemes:
  "w8a8"   int8, one fp32 scale per tensor, activations quantized per row to
           int8 inside the GEMV (the reference engine's own arithmetic)
  "q8g32"  int8 codes with an fp16 scale per 32 columns, fp32 activations
  "q4g64"  unsigned 4-bit codes with fp16 scale + zero per 64 columns
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field

import numpy as np

from . import _lib as L
from .ops import Context, Tensor, _dev_ptr, _stream_ptr


@dataclass(frozen=True)
class Geometry:
    hidden: int = 4096
    ffn: int = 12288
    vocab: int = 151936
    n_layers: int = 32
    attn_every: int = 4     # layer l is full attention when (l + 1) % attn_every == 0 (src/engine.zig:30-32)
    q_dim: int = 8192       # query + output gate
    kv_dim: int = 1024
    ssm_qkv: int = 6144     # Gated-DeltaNet q, k, v projection rows
    ssm_z: int = 2048       # Gated-DeltaNet gate projection rows
    eps: float = 1e-6
    head_dim: int = 0       # 0: reference stand-in out[i] = v[i % kv_dim]; else head-aligned GQA stand-in
    q_heads: int = 16
    kv_heads: int = 4
    # token mixers: "stub" -- the reference engine's stand-ins (src/engine.zig:619-623, :651-654);
    # "real" -- GQA attention with RoPE over a KV cache and the Gated-DeltaNet recurrence
    mixer: str = "stub"
    rope_theta: float = 1e6   # src/chpe_engine.zig:103
    ssm_heads: int = 16       # Gated-DeltaNet heads; key and value dims follow from ssm_qkv / ssm_z
    max_seq: int = 2048       # KV-cache positions ("real" mixers)

    def is_attn(self, l: int) -> bool:
        return (l + 1) % self.attn_every == 0

    @property
    def attn_hd(self) -> int:
        """Head dim of real attention: kv_dim / kv_heads."""
        return self.kv_dim // self.kv_heads

    @property
    def attn_gated(self) -> bool:
        """The q projection carries a per-head output gate after each head's
        query (Qwen3.5: q_dim = 2 x q_heads x head_dim)."""
        return self.q_dim == 2 * self.q_heads * self.attn_hd

    @property
    def ssm_dk(self) -> int:
        return (self.ssm_qkv - self.ssm_z) // (2 * self.ssm_heads)

    @property
    def ssm_dv(self) -> int:
        return self.ssm_z // self.ssm_heads

    def weight_count(self) -> int:
        H, F = self.hidden, self.ffn
        n = 0
        for l in range(self.n_layers):
            if self.is_attn(l):
                n += (self.q_dim + 2 * self.kv_dim) * H + H * H
            else:
                n += (self.ssm_qkv + self.ssm_z) * H + H * self.ssm_z
            n += 3 * F * H
        return n + self.vocab * H  # LM head (the embedding is a table lookup)


# Qwen3.5-9B hybrid: 24 Gated DeltaNet + 8 GQA layers, hidden 4096, FFN 12288,
# 16 q heads / 4 kv heads of 256, DeltaNet 16 heads of 128, vocab 151936.
QWEN35_9B = Geometry()
# Qwen2.5-72B: 80 GQA layers, hidden 8192, FFN 29568, 64 q / 8 kv heads of 128, vocab 152064.
QWEN25_72B = Geometry(hidden=8192, ffn=29568, vocab=152064, n_layers=80, attn_every=1, q_dim=8192, kv_dim=1024,
                      ssm_qkv=0, ssm_z=0, head_dim=128, q_heads=64, kv_heads=8)


@dataclass
class LayerWeights:
    in_gamma: object
    post_gamma: object
    proj: dict = field(default_factory=dict)  # name -> Tensor
    mix: dict = field(default_factory=dict)   # real mixers: Gated-DeltaNet conv taps and decays


SCHEMES = {"w8a8": (8, L.SCHEME_I8_TENSOR, 0), "q8g32": (8, L.SCHEME_I8_GROUP_F16, 32),
           "q4g64": (4, L.SCHEME_U_GROUP_F16_ZERO, 64)}


def quantize_device(ctx: Context, w, scheme: str):
    """Quantize fp32 device weights [rows, cols] with this library's quantizers.
    Returns (codes as packed row-major bytes, scales, zeros or None) on the device:
      w8a8  : s = max|w| / 127 over the tensor, q = clamp(rint(w / s), -127, 127)
      q8g32 : chpe_quantize_group_dev symmetric, group 32
      q4g64 : chpe_quantize_group_dev asymmetric 4-bit, group 64 (two codes per byte)"""
    import torch
    if scheme == "w8a8":
        m = w.abs().amax().float()
        s = torch.where(m > 1e-8, m / 127.0, torch.ones_like(m)).reshape(1)
        q = torch.clamp(torch.round(w / s), -127, 127).to(torch.int8)
        return q, s.float(), None
    bits, _, group = SCHEMES[scheme]
    codes, scales, zeros = ctx.quantize_group_dev(w, bits, group, symmetric=(scheme == "q8g32"))
    if bits == 4:
        codes = (codes[:, 0::2] | (codes[:, 1::2] << 4)).contiguous()
    return codes, scales, zeros


def upload_quantized(ctx: Context, codes, scales, zeros, scheme: str, rows: int, cols: int) -> Tensor:
    bits, sch, group = SCHEMES[scheme]
    return ctx.upload_matrix(bits, sch, codes, scales, zeros, rows=rows, cols=cols, group=group)


def build_random(ctx: Context, geom: Geometry, scheme: str, seed: int = 0, max_rows: int = 8, keep_host=False,
                 shard=None):
    """Random-init model (weights N(0, 0.02), quantized with `scheme`; norm
    gammas 1 + N(0, 0.02); int8 embedding table with one scale), built on the
    device.  `shard` = (rank, world) builds the tensor-parallel shard of that
    rank (column-split q/k/v/gate/up and LM head, row-split o/down).  With
    keep_host the quantized codes/scales are also returned as numpy arrays
    (for the oracle) in a dict keyed like the reference tensor map."""
    import torch
    gen = torch.Generator(device=f"cuda:{ctx.device}")
    gen.manual_seed(seed)
    dev = torch.device("cuda", ctx.device)
    eng = HybridEngine(ctx, geom, scheme, max_rows=max_rows)
    host = {} if keep_host else None
    rank, world = shard or (0, 1)
    H, F = geom.hidden, geom.ffn

    def mat(name, rows, cols, split=None):
        # the full matrix is drawn in 1 GiB row blocks so every shard sees the same weights
        w = torch.empty(rows, cols, device=dev)
        step = max(1, (1 << 28) // cols)
        for r0 in range(0, rows, step):
            r1 = min(rows, r0 + step)
            w[r0:r1].normal_(0.0, 0.02, generator=gen)
        if split == "col":
            w = w[rank * rows // world:(rank + 1) * rows // world]
        elif split == "ffn":  # rows of gate/up follow the down projection's K split
            w = w[_row_split(rows, world, rank, scheme)]
        elif split == "row":
            w = w[:, _row_split(cols, world, rank, scheme)]
        w = w.contiguous()
        codes, scales, zeros = quantize_device(ctx, w, scheme)
        t = upload_quantized(ctx, codes, scales, zeros, scheme, w.shape[0], w.shape[1])
        if host is not None:
            host[name] = (codes.cpu().numpy(), scales.cpu().numpy(), None if zeros is None else zeros.cpu().numpy())
        del w, codes, scales, zeros
        return t

    def gamma(name):
        v = (1.0 + 0.02 * torch.randn(H, device=dev, generator=gen)).float().contiguous()
        if host is not None:
            host[name] = v.cpu().numpy()
        return v

    emb = torch.empty(geom.vocab, H, device=dev).normal_(0.0, 0.02, generator=gen)
    es = float(emb.abs().amax() / 127.0)
    eng.embed = torch.clamp(torch.round(emb / es), -127, 127).to(torch.int8).contiguous()
    eng.embed_scale = es
    del emb
    if host is not None:
        host["embed"] = (eng.embed.cpu().numpy(), np.float32(es))
    tp = "col" if world > 1 else None
    for l in range(geom.n_layers):
        lw = LayerWeights(gamma(f"L{l}.in_gamma"), gamma(f"L{l}.post_gamma"))
        if geom.is_attn(l):
            lw.proj["q"] = mat(f"L{l}.q", geom.q_dim, H, tp)
            lw.proj["k"] = mat(f"L{l}.k", geom.kv_dim, H, tp)
            lw.proj["v"] = mat(f"L{l}.v", geom.kv_dim, H, tp)
            lw.proj["o"] = mat(f"L{l}.o", H, H, "row" if world > 1 else None)
        else:
            lw.proj["qkv"] = mat(f"L{l}.qkv", geom.ssm_qkv, H, tp)
            lw.proj["z"] = mat(f"L{l}.z", geom.ssm_z, H, tp)
            lw.proj["out"] = mat(f"L{l}.out", H, geom.ssm_z, "row" if world > 1 else None)
            if geom.mixer == "real":
                lw.mix = _delta_weights(geom, gen, dev)
                if host is not None:
                    host[f"L{l}.conv_w"] = lw.mix["conv_w"].cpu().numpy()
                    host[f"L{l}.decay"] = lw.mix["decay"].cpu().numpy()
        lw.proj["gate"] = mat(f"L{l}.gate", F, H, "ffn" if world > 1 else None)
        lw.proj["up"] = mat(f"L{l}.up", F, H, "ffn" if world > 1 else None)
        lw.proj["down"] = mat(f"L{l}.down", H, F, "row" if world > 1 else None)
        eng.layers.append(lw)
    eng.final_gamma = gamma("final_gamma")
    eng.head = mat("head", geom.vocab, H, tp)
    eng.init_mixer_state()
    torch.cuda.synchronize(dev)
    return eng, host


def build_random_codes(ctx: Context, geom: Geometry, scheme: str, seed: int = 0, max_rows: int = 8, shard=None):
    """Random-init model drawn directly in the quantized format (uniform codes,
    group scales drawn like those of quantized N(0, 0.02) weights), built shard
    by shard on the device.  Used for the large benchmark models, where drawing
    and quantizing ~70 G fp32 weights per rank would dominate start-up; the
    per-step work is the same as for build_random."""
    import torch
    dev = torch.device("cuda", ctx.device)
    rank, world = shard or (0, 1)
    gen = torch.Generator(device=dev)
    gen.manual_seed(seed * 1000 + rank)
    eng = HybridEngine(ctx, geom, scheme, max_rows=max_rows)
    bits, _, group = SCHEMES[scheme]
    H, F = geom.hidden, geom.ffn

    def mat(rows, cols):
        if scheme == "w8a8":
            codes = torch.randint(-127, 128, (rows, cols), dtype=torch.int8, device=dev, generator=gen)
            return upload_quantized(ctx, codes, torch.tensor([0.02 / 127 * 3], device=dev), None, scheme, rows, cols)
        codes = torch.randint(0, 256, (rows, cols * bits // 8), dtype=torch.uint8, device=dev, generator=gen)
        ng = cols // group
        base = 0.02 * 5.0 / ((1 << bits) - 1)  # range of ~5 sigma over the code range
        scales = (base * torch.exp(0.25 * torch.randn(rows, ng, device=dev, generator=gen))).half()
        zeros = None
        if scheme == "q4g64":
            zeros = torch.randint(6, 10, (rows, ng), device=dev, generator=gen).half()
        return upload_quantized(ctx, codes, scales, zeros, scheme, rows, cols)

    def split_rows(total, kind):
        if world == 1:
            return total
        if kind == "ffn":
            a, b = _row_split(total, world, rank, scheme).start, _row_split(total, world, rank, scheme).stop
            return b - a
        return (rank + 1) * total // world - rank * total // world

    def split_cols(total):
        if world == 1:
            return total
        sl = _row_split(total, world, rank, scheme)
        return sl.stop - sl.start

    gam = lambda: (1.0 + 0.02 * torch.randn(H, device=dev, generator=gen)).float().contiguous()
    eng.embed = torch.randint(-127, 128, (geom.vocab, H), dtype=torch.int8, device=dev, generator=gen)
    eng.embed_scale = 0.02 * 3 / 127
    for l in range(geom.n_layers):
        lw = LayerWeights(gam(), gam())
        if geom.is_attn(l):
            lw.proj["q"] = mat(split_rows(geom.q_dim, "col"), H)
            lw.proj["k"] = mat(split_rows(geom.kv_dim, "col"), H)
            lw.proj["v"] = mat(split_rows(geom.kv_dim, "col"), H)
            lw.proj["o"] = mat(H, split_cols(H))
        else:
            lw.proj["qkv"] = mat(split_rows(geom.ssm_qkv, "col"), H)
            lw.proj["z"] = mat(split_rows(geom.ssm_z, "col"), H)
            lw.proj["out"] = mat(H, split_cols(geom.ssm_z))
            if geom.mixer == "real":
                lw.mix = _delta_weights(geom, gen, dev)
        fr = split_rows(F, "ffn")
        lw.proj["gate"] = mat(fr, H)
        lw.proj["up"] = mat(fr, H)
        lw.proj["down"] = mat(H, split_cols(F))
        eng.layers.append(lw)
    eng.final_gamma = gam()
    eng.head = mat(split_rows(geom.vocab, "col"), H)
    eng.init_mixer_state()
    torch.cuda.synchronize(dev)
    return eng


def _delta_weights(geom: Geometry, gen, dev) -> dict:
    """Gated-DeltaNet weights of one layer (random init): depthwise conv1d taps
    [channels][4] ~ N(0, 0.3^2) and one decay per head, uniform in [0.5, 0.95]."""
    import torch
    C = geom.ssm_qkv
    conv_w = (0.3 * torch.randn(C, 4, device=dev, generator=gen)).float().contiguous()
    decay = (0.5 + 0.45 * torch.rand(geom.ssm_heads, device=dev, generator=gen)).float().contiguous()
    return {"conv_w": conv_w, "decay": decay}


def _row_split(cols: int, world: int, rank: int, scheme: str):
    """Columns of a row-split (K-split) projection owned by `rank`: contiguous,
    on group boundaries (64 for 4-bit, 32 for 8-bit) so no group is cut."""
    g = SCHEMES[scheme][2] or 32
    ng = cols // g
    a = rank * ng // world
    b = (rank + 1) * ng // world
    return slice(a * g, b * g)


class HybridEngine:
    """One model instance on one GPU (or one tensor-parallel shard; see tp.py)."""

    def __init__(self, ctx: Context, geom: Geometry, scheme: str, max_rows: int = 8):
        import torch
        self.ctx, self.geom, self.scheme, self.max_rows = ctx, geom, scheme, max_rows
        self.dev = torch.device("cuda", ctx.device)
        self.layers: list[LayerWeights] = []
        self.final_gamma = None
        self.embed = None          # int8 [vocab, hidden]
        self.embed_scale = 1.0
        self.head: Tensor | None = None
        self.graphs = {}
        self.xfrags = {}           # (input, rows) -> XFrag
        self.allreduce = None      # set by tensor parallelism: fn(tensor) summing across ranks (NCCL)
        self.comm = None           # or the NVLink one-shot all-reduce (ops.Comm)
        self.fuse_fills = False    # GEMVs build their own fragments (chpe_gemv_src_dev) instead of a shared fill
        self.fuse_exchange = True  # tensor parallel: the all-reduce runs inside the next RMSNorm fill
        self.push_exchange = False  # ... and the O / down GEMV sends the partials (the fill only collects)
        g, Mx = geom, max_rows
        f32 = dict(dtype=torch.float32, device=self.dev)
        widest = max(g.hidden, g.q_dim, g.ssm_qkv or 1, g.ffn)
        self.buf = {
            "hidden": torch.zeros(Mx, g.hidden, **f32), "norm": torch.zeros(Mx, g.hidden, **f32),
            "a": torch.zeros(Mx, widest, **f32), "b": torch.zeros(Mx, max(g.kv_dim, g.ssm_z, g.ffn), **f32),
            "c": torch.zeros(Mx, max(g.kv_dim, g.ffn), **f32), "mix": torch.zeros(Mx, g.hidden, **f32),
            "logits": torch.zeros(Mx, g.vocab, **f32), "tokens": torch.zeros(Mx, dtype=torch.int32, device=self.dev),
            "argmax": torch.zeros(Mx, dtype=torch.int32, device=self.dev), "maxv": torch.zeros(Mx, **f32),
            "mix_out": torch.zeros(Mx, g.hidden, **f32),
        }
        self.pos = torch.zeros(1, dtype=torch.int32, device=self.dev)  # positions cached (real mixers)
        self.mstate = {}  # layer -> {"kc", "vc"} or {"ring", "state"}

    # -- mixer state (real mixers) ----------------------------------------------------
    def init_mixer_state(self):
        """KV caches of the attention layers ([max_seq][local kv heads][head_dim]
        fp32) and the conv rings / recurrent states of the Gated-DeltaNet layers."""
        import torch
        g = self.geom
        if g.mixer != "real":
            return
        f32 = dict(dtype=torch.float32, device=self.dev)
        for l, lw in enumerate(self.layers):
            if "q" in lw.proj:
                kvh = lw.proj["k"].rows // g.attn_hd
                self.mstate[l] = {"kc": torch.zeros(g.max_seq, kvh, g.attn_hd, **f32),
                                  "vc": torch.zeros(g.max_seq, kvh, g.attn_hd, **f32)}
            else:
                self.mstate[l] = {"ring": torch.zeros(16, g.ssm_qkv, **f32),
                                  "state": torch.zeros(g.ssm_heads, g.ssm_dk, g.ssm_dv, **f32)}

    def reset(self):
        """Empty sequence: position 0, zero recurrent states and conv rings."""
        self.pos.zero_()
        for st in self.mstate.values():
            if "state" in st:
                st["state"].zero_()
                st["ring"].zero_()

    def _snapshot(self):
        return self.pos.clone(), {l: {k: v.clone() for k, v in st.items() if k != "kc" and k != "vc"}
                                  for l, st in self.mstate.items()}

    def _restore(self, snap):
        pos, st = snap
        self.pos.copy_(pos)
        for l, d in st.items():
            for k, v in d.items():
                self.mstate[l][k].copy_(v)

    # -- weights ---------------------------------------------------------------
    def n_weight_bytes(self) -> int:
        b = sum(t.device_bytes for lw in self.layers for t in lw.proj.values())
        return b + (self.head.device_bytes if self.head else 0)

    def _check(self, rc):
        self.ctx._check(rc)

    # -- one step ----------------------------------------------------------------
    def _xf(self, key: str, like: Tensor, M: int):
        """Activation fragments for the GEMVs of one input (created once per
        row count; filled once per step and read by every GEMV of that input)."""
        k = (key, M)
        if k not in self.xfrags:
            self.xfrags[k] = self.ctx.xfrag(like, M, L.X_F32)
        return self.xfrags[k]

    def step(self, M: int, stream=None):
        """Run one step over rows 0..M-1 of buf["tokens"]; leaves logits, argmax, maxv.

        Each GEMV input is produced straight into the MMA operand layout by one
        fused fill (RMSNorm of the hidden state, the token-mixer stand-ins, SiLU
        * mul), shared by the GEMVs of that input, so the normalised hidden
        state and the mixer outputs never reach memory; the Q/K/V (or DeltaNet
        qkv/z) projections share one launch, gate/up another.  With fuse_fills
        each GEMV builds its fragments in its own CTAs instead."""
        import torch
        g, ctx, lib = self.geom, self.ctx, self.ctx.lib
        b = self.buf
        st = stream or torch.cuda.current_stream(self.dev)
        sp = _stream_ptr(st)
        H = g.hidden
        # fused fills only on request: every CTA of a K-slice builds the same
        # fragments, which on B200 costs more than the fill kernel it saves
        fused = self.fuse_fills and self.scheme != "w8a8"

        pending = []  # a tensor-parallel partial whose all-reduce is due before hidden is next read

        def flush():
            if pending:  # (a pushing GEMV's partial is sent again: the same words under the same epoch)
                self.comm.allreduce_residual(pending.pop()[0], b["hidden"], M * H, stream=sp.value)

        def run(ts, ys, op, x, aux=None, mode=0, acc=False, push=False, **kw):
            """ys (+)= op(x, aux) . W^T for the tensors ts (one launch); push:
            the GEMV also sends its outputs to the peers for the next exchange
            (returns whether it did)."""
            if fused:
                flush()
                ctx.gemv_src(ts, ys, op, x, aux, M=M, mode=mode, accumulate=acc, stream=sp.value, **kw)
                return False
            xf = self._xf(("in", ts[0].cols), ts[0], M)
            if pending and op == L.XOP_RMSNORM and x is b["hidden"] and \
                    self.comm.allreduce_fill(pending[-1][0], x, xf, aux, kw.get("eps", 0.0), stream=sp.value,
                                             pushed=pending[-1][1]):
                pending.pop()  # the all-reduce ran inside the RMSNorm fill
            else:
                flush()
                ctx.xfrag_fill_op(xf, op, x, aux, stream=sp.value, **kw)
            if push and self.comm.gemv_push(ts[0], xf, ys[0], stream=sp.value):
                return True
            if mode == 1:
                self._check(lib.chpe_gemv_gateup_swiglu_xfrag_dev(ctx.ptr, ts[0].handle, ts[1].handle, xf.handle,
                                                                  _dev_ptr(ys[0]), sp))
            elif len(ts) > 1:
                ctx.gemv_multi_xfrag(ts, xf, ys, stream=sp.value)
            else:
                ctx.gemv_xfrag(ts[0], xf, ys[0], accumulate=acc, stream=sp.value)

        def run_res(t: Tensor, op, x, aux=None, **kw):
            """hidden += op(x) . W^T (the residual add of the block); with tensor
            parallelism the shard's partial sum is summed over the ranks first:
            inside the next RMSNorm fill of hidden (comm, fuse_exchange; with
            push_exchange the GEMV itself sends the partial), by the one-shot
            NVLink all-reduce kernel, or by an NCCL all-reduce and an add."""
            hidden = b["hidden"]
            if self.comm is None and self.allreduce is None:
                run([t], [hidden], op, x, aux, acc=True, **kw)
                return
            part = b["mix_out"][:M]
            pushed = bool(run([t], [part], op, x, aux, push=self.comm is not None and self.fuse_exchange and
                              self.push_exchange, **kw))
            if self.comm is not None:
                if self.fuse_exchange:
                    pending.append((part, pushed))  # summed by the next RMSNorm fill of hidden
                else:
                    self.comm.allreduce_residual(part, hidden, M * H, stream=sp.value)
            else:
                self.allreduce(part)
                hidden[:M].add_(part)

        self._check(lib.chpe_embed_i8_dev(ctx.ptr, _dev_ptr(self.embed), C.c_float(self.embed_scale), H, g.vocab,
                                          _dev_ptr(b["tokens"]), M, _dev_ptr(b["hidden"]), sp))
        hid = b["hidden"]
        norm = dict(ldx=H, eps=g.eps)
        real = g.mixer == "real"
        for l, lw in enumerate(self.layers):
            p = lw.proj
            if "q" in p and real:  # full attention: RoPE, KV cache, GQA softmax attention
                q_out, k_out, v_out, att = b["a"], b["b"], b["c"], b["mix"]
                run([p["q"], p["k"], p["v"]], [q_out, k_out, v_out], L.XOP_RMSNORM, hid, lw.in_gamma, **norm)
                hd = g.attn_hd
                kvh = p["k"].rows // hd
                qh = p["q"].rows // (hd * (2 if g.attn_gated else 1))
                ms = self.mstate[l]
                ctx.attn_decode(q_out, k_out, v_out, ms["kc"], ms["vc"], self.pos, M, qh, kvh, hd, g.rope_theta,
                                g.attn_gated, att, ldq=p["q"].rows, ldkv=p["k"].rows, ldo=qh * hd, stream=sp.value)
                run_res(p["o"], L.XOP_PLAIN, att, ldx=qh * hd)
            elif "q" in p:  # full attention (GQA) block; stand-in mixer = V broadcast
                q_out, k_out, v_out = b["a"], b["b"], b["c"]
                kv = p["v"].rows
                run([p["q"], p["k"], p["v"]], [q_out, k_out, v_out], L.XOP_RMSNORM, hid, lw.in_gamma, **norm)
                run_res(p["o"], L.XOP_ATTN_STUB, v_out, ldx=kv, kv_dim=kv, head_dim=g.head_dim,
                        group=g.q_heads // g.kv_heads)
            elif real:  # Gated DeltaNet: conv1d + recurrence, output gated by silu(z)
                qkv_out, z_out, y = b["a"], b["b"], b["mix"]
                run([p["qkv"], p["z"]], [qkv_out, z_out], L.XOP_RMSNORM, hid, lw.in_gamma, **norm)
                ms = self.mstate[l]
                ctx.deltanet_step(qkv_out, lw.mix["conv_w"], ms["ring"], ms["state"], lw.mix["decay"], self.pos, M,
                                  g.ssm_heads, g.ssm_dk, g.ssm_dv, y, ldqkv=p["qkv"].rows, ldo=g.ssm_z,
                                  stream=sp.value)
                run_res(p["out"], L.XOP_SSM_STUB, y, z_out, ldx=g.ssm_z, ld_aux=p["z"].rows, qkv_dim=g.ssm_z,
                        silu_on_qkv=False)
            else:  # Gated DeltaNet block; stand-in mixer = qkv gated by z
                qkv_out, z_out = b["a"], b["b"]
                run([p["qkv"], p["z"]], [qkv_out, z_out], L.XOP_RMSNORM, hid, lw.in_gamma, **norm)
                run_res(p["out"], L.XOP_SSM_STUB, qkv_out, z_out, ldx=p["qkv"].rows, ld_aux=p["z"].rows,
                        qkv_dim=p["qkv"].rows, silu_on_qkv=M > 1)
            if M == 1:  # src/engine.zig:682 fused gate/up SwiGLU
                run([p["gate"], p["up"]], [b["a"]], L.XOP_RMSNORM, hid, lw.post_gamma, mode=1, **norm)
                run_res(p["down"], L.XOP_PLAIN, b["a"], ldx=p["down"].cols)
            else:  # src/engine.zig:839-844 unfused gate, up, siluMul
                run([p["gate"], p["up"]], [b["b"], b["c"]], L.XOP_RMSNORM, hid, lw.post_gamma, **norm)
                run_res(p["down"], L.XOP_SILU_MUL, b["b"], b["c"], ldx=p["gate"].rows, ld_aux=p["up"].rows)
        run([self.head], [b["logits"]], L.XOP_RMSNORM, hid, self.final_gamma, **norm)
        flush()
        self._check(lib.chpe_argmax_dev(ctx.ptr, _dev_ptr(b["logits"]), M, self.head.rows, _dev_ptr(b["argmax"]),
                                        _dev_ptr(b["maxv"]), sp))
        if real:
            ctx.pos_advance(self.pos, M, stream=sp.value)

    def capture(self, M: int):
        """Capture step(M) as a CUDA graph (after one eager warm-up run, whose
        effect on the position, recurrent states and conv rings is undone)."""
        import torch
        snap = self._snapshot()
        st = torch.cuda.Stream(self.dev)
        st.wait_stream(torch.cuda.current_stream(self.dev))
        with torch.cuda.stream(st):
            self.step(M, st)
        torch.cuda.synchronize(self.dev)
        self._restore(snap)
        torch.cuda.synchronize(self.dev)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=st):
            self.step(M, st)
        self.graphs[M] = g
        return g

    def prefill(self, tokens, M: int = 8, use_graph: bool = True):
        """Feed a context through the step, M positions at a time (the verify
        step; with real mixers this fills the KV caches and recurrent states).
        A last partial chunk runs eagerly with its own row count."""
        import torch
        b = self.buf
        toks = np.asarray(tokens, np.int32)
        if use_graph and M not in self.graphs:
            self.capture(M)
        i = 0
        while i < len(toks):
            n = min(M, len(toks) - i)
            b["tokens"][:n].copy_(torch.from_numpy(toks[i:i + n]).to(self.dev))
            if n == M and use_graph:
                self.graphs[M].replay()
            else:
                self.step(n)
            i += n
        torch.cuda.synchronize(self.dev)

    def decode_greedy(self, first_tokens, steps: int, M: int = 1, use_graph: bool = True):
        """Greedy decode: each step's argmax rows become the next step's tokens.
        Returns the argmax tokens of every step as an int array [steps, M]."""
        import torch
        b = self.buf
        b["tokens"][:M].copy_(torch.as_tensor(np.asarray(first_tokens, np.int32)[:M], device=self.dev))
        out = torch.empty(steps, M, dtype=torch.int32, device=self.dev)
        if use_graph and M not in self.graphs:
            self.capture(M)
            b["tokens"][:M].copy_(torch.as_tensor(np.asarray(first_tokens, np.int32)[:M], device=self.dev))
        for s in range(steps):
            if use_graph:
                self.graphs[M].replay()
            else:
                self.step(M)
            out[s].copy_(b["argmax"][:M])
            b["tokens"][:M].copy_(b["argmax"][:M])
        torch.cuda.synchronize(self.dev)
        return out.cpu().numpy()
