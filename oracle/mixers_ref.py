"""CPU restatement of the reference's token mixers (numpy, float32).

TEST INFRASTRUCTURE ONLY (the oracle): used by tests/ and the oracle engine.

* apply_rope: src/qwen72b_engine.zig:90-111 / src/chpe_engine.zig:191-212
  (pair i with i + head_dim/2; freq = 1 / theta^(2i/head_dim); angle = p *
  freq).  pow, cos and sin are taken in float64 and rounded to float32 -- the
  reference's f32 math functions are not reproducible bit for bit across
  libraries, and the CUDA path does the same, so both agree exactly.
* attention: src/qwen72b_engine.zig:291-369 / src/chpe_engine.zig:690-745 --
  write the rotated key and the value at the position, then per query head
  (kv head = head / group) scores dot(q, k_t) * 1/sqrt(head_dim) over
  t = 0 .. position, softmax with the maximum subtracted, weights times
  1/sum, weighted sum of the values.  The optional output gate (Qwen3.5's
  q projection carries head_dim gate values after each head's query):
  out * sigmoid(gate).
* conv1d: src/ssm.zig:11-41 Conv1DRingBuffer (width 4; tap k weighs the input
  k positions back, summed k = 0..3 in order).
* linear attention: src/ssm.zig:45-99 LinearAttentionState.update
  (S = S * decay + k^T v, elementwise in that order; y = q S).
"""
from __future__ import annotations

import numpy as np

f32 = np.float32


def rope_cs(head_dim: int, theta: float, p: int):
    i = np.arange(head_dim // 2)
    e = (f32(2.0) * i.astype(f32)) / f32(head_dim)
    freq = f32(1.0) / np.power(np.float64(np.float32(theta)), e.astype(np.float64)).astype(f32)
    ang = f32(p) * freq
    return np.cos(ang.astype(np.float64)).astype(f32), np.sin(ang.astype(np.float64)).astype(f32)


def apply_rope(vec, p: int, n_heads: int, head_dim: int, theta: float):
    """src/qwen72b_engine.zig:90-111: rotates every head of vec (float32) at position p."""
    out = np.array(vec, f32).reshape(n_heads, head_dim).copy()
    c, s = rope_cs(head_dim, theta, p)
    h = head_dim // 2
    v0, v1 = out[:, :h].copy(), out[:, h:].copy()
    out[:, :h] = v0 * c - v1 * s
    out[:, h:] = v0 * s + v1 * c
    return out.reshape(-1)


def sigmoid(x):
    x = np.asarray(x, f32)
    return (f32(1.0) / (f32(1.0) + np.exp(-x.astype(np.float64)).astype(f32))).astype(f32)


class AttnLayerRef:
    """KV cache of one attention layer, [max_seq][kv_heads][head_dim] float32."""

    def __init__(self, max_seq, q_heads, kv_heads, head_dim, theta, gated):
        self.kc = np.zeros((max_seq, kv_heads, head_dim), f32)
        self.vc = np.zeros((max_seq, kv_heads, head_dim), f32)
        self.qh, self.kvh, self.hd, self.theta, self.gated = q_heads, kv_heads, head_dim, theta, gated

    def step(self, q_rows, k_rows, v_rows, pos: int):
        """Rows m = 0..M-1 at positions pos + m (causal); returns [M][q_heads*head_dim]."""
        qh, kvh, hd = self.qh, self.kvh, self.hd
        grp = qh // kvh
        scale = f32(1.0) / f32(np.sqrt(f32(hd)))
        outs = []
        for m in range(len(q_rows)):
            p = pos + m
            qr = np.asarray(q_rows[m], f32)
            if self.gated:
                qg = qr[:qh * 2 * hd].reshape(qh, 2, hd)
                qq, gate = qg[:, 0].reshape(-1), qg[:, 1].reshape(-1)
            else:
                qq, gate = qr[:qh * hd], None
            q = apply_rope(qq, p, qh, hd, self.theta).reshape(qh, hd)
            self.kc[p] = apply_rope(np.asarray(k_rows[m], f32)[:kvh * hd], p, kvh, hd, self.theta).reshape(kvh, hd)
            self.vc[p] = np.asarray(v_rows[m], f32)[:kvh * hd].reshape(kvh, hd)
            # every query head at once (head h reads kv head h // grp)
            K = self.kc[:p + 1].reshape(p + 1, kvh, 1, hd)
            V = self.vc[:p + 1].reshape(p + 1, kvh, 1, hd)
            qg = q.reshape(kvh, grp, hd)
            sc = np.einsum("tjd,jgd->jgt", K[:, :, 0, :], qg).astype(f32) * scale  # [kvh, grp, t]
            e = np.exp(sc - sc.max(axis=-1, keepdims=True)).astype(f32)
            w = e * (f32(1.0) / e.sum(axis=-1, keepdims=True, dtype=f32))
            out = np.einsum("jgt,tjd->jgd", w, V[:, :, 0, :]).astype(f32).reshape(qh, hd)
            if gate is not None:
                out = out * sigmoid(gate).reshape(qh, hd)
            outs.append(out.reshape(-1))
        return np.stack(outs).astype(f32)


class DeltaLayerRef:
    """Conv ring (per channel, the last inputs) and state [heads][key_dim][value_dim]."""

    def __init__(self, heads, key_dim, value_dim, conv_w, decay):
        self.H, self.dk, self.dv = heads, key_dim, value_dim
        self.C = heads * (2 * key_dim + value_dim)
        self.w = np.asarray(conv_w, f32).reshape(self.C, 4)
        self.decay = np.asarray(decay, f32)
        self.hist = []  # inputs of earlier positions, newest last
        self.S = np.zeros((heads, key_dim, value_dim), f32)

    def conv(self, x):
        """src/ssm.zig:26-41 with x the newest input: sum over taps k = 0..3 of input(t - k) * w[:, k]."""
        taps = [x] + [self.hist[-k] if k <= len(self.hist) else np.zeros(self.C, f32) for k in range(1, 4)]
        s = np.zeros(self.C, f32)
        for k in range(4):
            s = (s + taps[k] * self.w[:, k]).astype(f32)
        return s

    def step(self, qkv_rows):
        H, dk, dv = self.H, self.dk, self.dv
        outs = []
        for row in qkv_rows:
            x = np.asarray(row, f32)[:self.C]
            c = self.conv(x)
            self.hist.append(x.copy())
            self.hist = self.hist[-3:]
            q = c[:H * dk].reshape(H, dk)
            k = c[H * dk:2 * H * dk].reshape(H, dk)
            v = c[2 * H * dk:].reshape(H, dv)
            y = np.zeros((H, dv), f32)
            for h in range(H):  # src/ssm.zig:70-98
                self.S[h] = (self.S[h] * self.decay[h] + np.outer(k[h], v[h]).astype(f32)).astype(f32)
                y[h] = (q[h] @ self.S[h]).astype(f32)
            outs.append(y.reshape(-1))
        return np.stack(outs).astype(f32)
