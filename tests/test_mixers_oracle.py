"""The oracle's token mixers (oracle/mixers_ref.py) against literal,
loop-by-loop restatements of the reference functions at small sizes: the
vectorised oracle must agree with the reference's own loop order (these run
on the CPU, no GPU needed).

* attention: src/qwen72b_engine.zig:291-369 (per query head: scores t = 0..pos,
  max, exp, 1/sum, weighted value sum) and applyRope :90-111;
* conv1d ring buffer: src/ssm.zig:11-41 (a 4-slot ring with a head index:
  step writes history[head] and advances it; convolve reads
  history[(head + 3 - k) % 4] for tap k);
* the recurrence: src/ssm.zig:70-98.
"""
import numpy as np

from oracle.mixers_ref import AttnLayerRef, DeltaLayerRef, apply_rope, rope_cs

f32 = np.float32


def test_rope_pairs_and_position_zero():
    v = np.arange(16, dtype=f32)
    assert np.array_equal(apply_rope(v, 0, 2, 8, 1e6), v)  # angle 0: identity
    c, s = rope_cs(8, 1e6, 5)
    out = apply_rope(v, 5, 2, 8, 1e6).reshape(2, 8)
    for h in range(2):
        for i in range(4):
            v0, v1 = v[h * 8 + i], v[h * 8 + i + 4]
            assert out[h, i] == f32(f32(v0 * c[i]) - f32(v1 * s[i]))
            assert out[h, i + 4] == f32(f32(v0 * s[i]) + f32(v1 * c[i]))


def test_attention_matches_reference_loops():
    rng = np.random.default_rng(0)
    qh, kvh, hd, theta = 4, 2, 8, 1e6
    ref = AttnLayerRef(16, qh, kvh, hd, theta, False)
    kc = np.zeros((16, kvh * hd), f32)
    vc = np.zeros((16, kvh * hd), f32)
    for pos in range(6):
        q = rng.standard_normal(qh * hd).astype(f32)
        k = rng.standard_normal(kvh * hd).astype(f32)
        v = rng.standard_normal(kvh * hd).astype(f32)
        got = ref.step(q[None], k[None], v[None], pos)[0]
        # literal restatement of forwardDecode's attention
        qr = apply_rope(q, pos, qh, hd, theta)
        kc[pos] = apply_rope(k, pos, kvh, hd, theta)
        vc[pos] = v
        out = np.zeros(qh * hd, f32)
        scale = f32(1.0) / f32(np.sqrt(f32(hd)))
        for h in range(qh):
            j = h // (qh // kvh)
            scores = np.zeros(pos + 1, f32)
            mx = f32(-1e30)
            for t in range(pos + 1):
                d = f32(0.0)
                for x in range(hd):
                    d = f32(d + f32(qr[h * hd + x] * kc[t, j * hd + x]))
                scores[t] = f32(d * scale)
                mx = max(mx, scores[t])
            se = f32(0.0)
            for t in range(pos + 1):
                scores[t] = f32(np.exp(f32(scores[t] - mx)))
                se = f32(se + scores[t])
            inv = f32(f32(1.0) / se)
            for t in range(pos + 1):
                w = f32(scores[t] * inv)
                for x in range(hd):
                    out[h * hd + x] = f32(out[h * hd + x] + f32(w * vc[t, j * hd + x]))
        assert np.allclose(got, out, rtol=1e-5, atol=1e-6)
        assert np.array_equal(ref.kc[pos].reshape(-1), kc[pos])


def test_deltanet_matches_reference_ring_and_update():
    rng = np.random.default_rng(1)
    H, dk, dv = 2, 4, 4
    C = H * (2 * dk + dv)
    w = rng.standard_normal((C, 4)).astype(f32)
    decay = np.array([0.9, 0.5], f32)
    ref = DeltaLayerRef(H, dk, dv, w, decay)
    hist = np.zeros((4, C), f32)  # the reference ring: 4 slots and a head index
    head = 0
    S = np.zeros((H, dk, dv), f32)
    for step in range(7):
        x = rng.standard_normal(C).astype(f32)
        got = ref.step(x[None])[0]
        hist[head] = x  # Conv1DRingBuffer.step
        head = (head + 1) % 4
        conv = np.zeros(C, f32)
        for c in range(C):  # Conv1DRingBuffer.convolve
            s = f32(0.0)
            for k in range(4):
                s = f32(s + f32(hist[(head + 4 - 1 - k) % 4][c] * w[c][k]))
            conv[c] = s
        q = conv[:H * dk].reshape(H, dk)
        kk = conv[H * dk:2 * H * dk].reshape(H, dk)
        v = conv[2 * H * dk:].reshape(H, dv)
        y = np.zeros((H, dv), f32)
        for h in range(H):  # LinearAttentionState.update
            for i in range(dk):
                for j in range(dv):
                    S[h, i, j] = f32(f32(S[h, i, j] * decay[h]) + f32(kk[h, i] * v[h, j]))
            for j in range(dv):
                acc = f32(0.0)
                for i in range(dk):
                    acc = f32(acc + f32(q[h, i] * S[h, i, j]))
                y[h, j] = acc
        assert np.array_equal(ref.S, S)
        assert np.allclose(got, y.reshape(-1), rtol=1e-5, atol=1e-6)
