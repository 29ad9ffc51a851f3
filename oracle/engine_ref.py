"""CPU restatement of the reference engine's decode / verify step.

TEST INFRASTRUCTURE ONLY (the oracle): used by tests/ to check the GPU engine.

Follows src/engine.zig Qwen35Engine: embedToken (:567-580), step (:583-734),
stepBatch4 (:753-900), stepBatch8 (:902-1095) and computeArgmax (:1098-1110),
with the reference's stand-in mixers (attention: V broadcast :619-623;
Gated DeltaNet: qkv * silu(z) at batch 1 :651-654, silu(qkv) * z at batch 4/8
:813/:988), or -- geometry mixer "real" -- the reference's attention with RoPE
and KV cache and its Gated-DeltaNet conv1d + recurrence (oracle/mixers_ref.py),
the DeltaNet output gated by silu(z); rows of a step are then consecutive
positions of one sequence.  The per-tensor int8 scheme uses the oracle's restatement of the
reference's own operators (gemvParallel / gemvGateUpSwiGLUParallel /
quantizeActivationInt8 / rmsnorm); the grouped schemes use the grouped GEMV
specification (fp64 accumulation) on fp32 activations.
"""
from __future__ import annotations

import os

import numpy as np

from oracle import oracle as O
from oracle.mixers_ref import AttnLayerRef, DeltaLayerRef


def _silu(x):
    """g / (1 + exp(-g)) in float32, exp taken in float64 and rounded to float32
    (as the oracle's C silu and the CUDA path do)."""
    x = np.asarray(x, np.float32)
    e = np.exp(-x.astype(np.float64)).astype(np.float32)
    return (x / (np.float32(1.0) + e)).astype(np.float32)


class EngineRef:
    def __init__(self, host: dict, geom, scheme: str, num_workers: int | None = None):
        self.h, self.g, self.scheme = host, geom, scheme
        self.nw = num_workers or os.cpu_count() or 8
        self._unpacked = {}  # q4g64: codes one per byte, made once per tensor
        self.pos = 0
        self.mix = {}
        if getattr(geom, "mixer", "stub") == "real":
            for l in range(geom.n_layers):
                if geom.is_attn(l):
                    self.mix[l] = AttnLayerRef(geom.max_seq, geom.q_heads, geom.kv_heads, geom.attn_hd,
                                               geom.rope_theta, geom.attn_gated)
                else:
                    self.mix[l] = DeltaLayerRef(geom.ssm_heads, geom.ssm_dk, geom.ssm_dv, host[f"L{l}.conv_w"],
                                                host[f"L{l}.decay"])

    # -- one projection: y[M, rows] = x[M, cols] . W^T ------------------------------
    def gemv(self, name, x):
        codes, scales, zeros = self.h[name]
        x = np.asarray(x, np.float32)
        if self.scheme == "w8a8":
            out = []
            for row in x:
                q, s = O.quantize_act_i8(row)
                out.append(O.gemv_parallel(codes, float(scales[0]), q, float(s), num_workers=self.nw))
            return np.stack(out)
        if self.scheme == "q8g32":
            return O.gemv_grouped(codes.view(np.int8), scales, None, 32, x, num_workers=self.nw)
        # q4g64: two codes per byte, low nibble first
        c = self._unpacked.get(name)
        if c is None:
            c = np.empty((codes.shape[0], codes.shape[1] * 2), np.uint8)
            c[:, 0::2] = codes & 0x0F
            c[:, 1::2] = codes >> 4
            self._unpacked[name] = c
        return O.gemv_grouped(c, scales, zeros, 64, x, num_workers=self.nw)

    def gateup(self, l, x):
        """Batch 1: fused gate/up SwiGLU (src/engine.zig:682)."""
        if self.scheme == "w8a8":
            (wg, sg, _), (wu, su, _) = self.h[f"L{l}.gate"], self.h[f"L{l}.up"]
            q, s = O.quantize_act_i8(x[0])
            return O.gemv_gateup_swiglu_parallel(wg, float(sg[0]), wu, float(su[0]), q, float(s),
                                                 num_workers=self.nw)[None]
        g = self.gemv(f"L{l}.gate", x)
        u = self.gemv(f"L{l}.up", x)
        return (_silu(g) * u).astype(np.float32)

    def step(self, tokens):
        g, h = self.g, self.h
        M = len(tokens)
        emb, es = h["embed"]
        hidden = np.stack([emb[t].astype(np.float32) * np.float32(es) for t in tokens]).astype(np.float32)
        norm = lambda x, name: np.stack([O.rmsnorm(r, h[name], g.eps) for r in x])
        for l in range(g.n_layers):
            x = norm(hidden, f"L{l}.in_gamma")
            if g.is_attn(l) and l in self.mix:
                q = self.gemv(f"L{l}.q", x)
                k = self.gemv(f"L{l}.k", x)
                v = self.gemv(f"L{l}.v", x)
                mix = self.mix[l].step(q, k, v, self.pos)
                hidden = (hidden + self.gemv(f"L{l}.o", mix)).astype(np.float32)
            elif l in self.mix:
                qkv = self.gemv(f"L{l}.qkv", x)
                z = self.gemv(f"L{l}.z", x)
                y = self.mix[l].step(qkv)
                hidden = (hidden + self.gemv(f"L{l}.out", (y * _silu(z)).astype(np.float32))).astype(np.float32)
            elif g.is_attn(l):
                self.gemv(f"L{l}.q", x)
                self.gemv(f"L{l}.k", x)
                v = self.gemv(f"L{l}.v", x)
                kv = v.shape[1]
                o_in = h[f"L{l}.o"][0].shape[1] * (2 if self.scheme == "q4g64" else 1)
                i = np.arange(o_in)
                if g.head_dim:  # head-aligned form: query head h of head_dim columns takes kv head h / group
                    hd, grp = g.head_dim, g.q_heads // g.kv_heads
                    mix = v[:, ((i // hd) // grp) * hd + i % hd]
                else:  # the reference's form, out[i] = v[i % kv_dim] (src/engine.zig:619-623)
                    mix = v[:, i % kv]
                hidden = (hidden + self.gemv(f"L{l}.o", mix)).astype(np.float32)
            else:
                qkv = self.gemv(f"L{l}.qkv", x)
                z = self.gemv(f"L{l}.z", x)
                n = z.shape[1]
                qq = qkv[:, np.arange(n) % qkv.shape[1]]
                mix = (qq * _silu(z)) if M == 1 else (_silu(qq) * z)
                hidden = (hidden + self.gemv(f"L{l}.out", mix.astype(np.float32))).astype(np.float32)
            x = norm(hidden, f"L{l}.post_gamma")
            if M == 1:
                mlp = self.gateup(l, x)
            else:
                gt = self.gemv(f"L{l}.gate", x)
                up = self.gemv(f"L{l}.up", x)
                mlp = np.stack([O.silu_mul(a, b) for a, b in zip(gt, up)])
            hidden = (hidden + self.gemv(f"L{l}.down", mlp)).astype(np.float32)
        x = norm(hidden, "final_gamma")
        logits = self.gemv("head", x)
        self.pos += M
        return [O.argmax(r)[0] for r in logits], logits

    def decode_greedy(self, first_tokens, steps):
        toks = list(first_tokens)
        out = []
        for _ in range(steps):
            nxt, _ = self.step(toks)
            out.append(nxt)
            toks = nxt
        return np.array(out, np.int32)
