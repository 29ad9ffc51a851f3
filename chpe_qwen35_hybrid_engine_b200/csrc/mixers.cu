// mixers.cu -- the token mixers of a decode / verify step: grouped-query
// attention over a KV cache with rotary position embeddings (the full-attention
// layers), and the Gated-DeltaNet linear-attention recurrence with its causal
// conv1d ring buffer (the linear-attention layers of the hybrid model).
//
// Rows of a step are consecutive positions of one sequence: row m of an
// M-row step sits at position pos + m, where pos (a device int, so a captured
// step replays at the right position) is the number of positions already in
// the cache; chpe_pos_advance_dev moves it on by M after the step.  Row m
// attends causally to positions 0 .. pos + m, and the recurrence consumes the
// rows in order.
//
// Attention (src/qwen72b_engine.zig:90-111 applyRope, :291-369 forwardDecode;
// src/chpe_engine.zig:191-212, :690-745): grid (kv head, split of 64
// positions).  A CTA stages the rotated queries of its kv head's group (all
// rows) and its 64 cached keys and values in shared memory -- writing the
// rotated keys and the values of the step's new positions into the cache when
// they fall in its split -- scores them (1/sqrt(head_dim)), and keeps a
// partial softmax (max, sum, weighted value sum) per query.  The last CTA of a
// kv head to finish (an arrival count) combines the splits in split order, so
// the result does not depend on scheduling.  KV cache: fp32
// [max_seq][kv_heads][head_dim] per layer, as the reference keeps it.
//
// Gated DeltaNet (src/ssm.zig:11-99): grid (head, 32-column slab of the value
// dimension).  Per row: the depthwise causal conv1d of width 4 over the
// q / k / v channels (Conv1DRingBuffer.convolve; the ring holds the last
// inputs per channel), then S = decay[h] * S + k^T v and y = q S
// (LinearAttentionState.update), the head's 128 x 128 state held in the
// registers of the CTA's 256 threads (16 rows each) across the step's rows.
#include <cfloat>

#include "../../include/chpe_b200.h"
#include "common.cuh"
#include "internal.h"
#include "xsrc.cuh"

namespace chpe {

constexpr int kAttnTc = 64;        // positions per attention CTA
constexpr int kAttnThreads = 256;
constexpr int kAttnMaxQ = 64;      // queries per CTA: group (q heads per kv head) x rows
constexpr int kRingSlots = 16;     // conv ring positions per channel (>= rows + 3)
constexpr int kConvWidth = 4;
constexpr int kErrCacheFull = 41;  // a step past the KV cache's max_seq positions

// RoPE factors of pair i of a head_dim-wide head at position p, as the
// reference computes them (f32: e = 2i / head_dim, freq = 1 / theta^e,
// angle = p * freq) with pow, cos and sin taken in double and rounded to
// float -- the oracle does the same, so both get the same bits.
__device__ __forceinline__ void rope_cs(int i, int head_dim, float theta, int p, float &c, float &s) {
    const float e = __fdiv_rn(2.0f * (float)i, (float)head_dim);
    const float freq = __fdiv_rn(1.0f, (float)pow((double)theta, (double)e));
    const float ang = __fmul_rn((float)p, freq);
    c = (float)cos((double)ang);
    s = (float)sin((double)ang);
}

struct AttnParams {
    const float *q;  // rows [M][ldq]: per q head, head_dim query values (then head_dim gate values when gated)
    const float *k, *v;  // rows [M][ldkv]: kv_heads x head_dim
    int ldq, ldkv;
    float *kc, *vc;  // this layer's cache [max_seq][kv_heads][head_dim]
    const int *pos;
    int M, qh, kvh, hd, max_seq, gated;
    float theta, scale;
    float *out;  // rows [M][ldo]: q_heads x head_dim
    int ldo;
    float *part;    // partials [kvh][nsplit][kAttnMaxQ][hd + 2]
    unsigned *ctr;  // arrivals per kv head (self-resetting)
    int nsplit;
    int *err;
};

__global__ void __launch_bounds__(kAttnThreads) chpe_attn_decode_kernel(const AttnParams p) {
    extern __shared__ __align__(16) float sm[];
    __shared__ unsigned s_last;
    pdl_begin();
    const int j = blockIdx.x;  // kv head
    const int sp = blockIdx.y;
    const int hd = p.hd, G = p.qh / p.kvh, NQ = G * p.M;
    const int pos = *p.pos;
    const int tmax = pos + p.M;  // positions after this step
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (pos < 0 || tmax > p.max_seq) {  // the cache is full: record it, touch nothing (every CTA returns)
        if (j == 0 && sp == 0 && tid == 0) atomicExch(p.err, kErrCacheFull);
        return;
    }
    const int t0 = sp * kAttnTc, t1 = min(t0 + kAttnTc, tmax);
    const int ldk = hd + 1;  // padded rows: lanes read different positions without bank conflicts
    float *qs = sm;                       // [NQ][hd]
    float *ks = qs + NQ * hd;             // [kAttnTc][hd + 1]
    float *vs = ks + kAttnTc * ldk;       // [kAttnTc][hd]
    float *ps = vs + kAttnTc * hd;        // [NQ][kAttnTc] probabilities
    const int qstride = p.gated ? 2 * hd : hd;
    if (t0 < t1) {
        // rotated queries: query qi = g * M + m is q head j * G + g of row m at position pos + m
        for (int e = tid; e < NQ * (hd / 2); e += kAttnThreads) {
            const int qi = e / (hd / 2), i = e % (hd / 2);
            const int g = qi / p.M, m = qi % p.M;
            const float *src = p.q + (size_t)m * p.ldq + (size_t)(j * G + g) * qstride;
            float c, s;
            rope_cs(i, hd, p.theta, pos + m, c, s);
            const float v0 = src[i], v1 = src[i + hd / 2];
            qs[qi * hd + i] = __fsub_rn(__fmul_rn(v0, c), __fmul_rn(v1, s));
            qs[qi * hd + i + hd / 2] = __fadd_rn(__fmul_rn(v0, s), __fmul_rn(v1, c));
        }
        // keys and values of positions t0 .. t1-1: cached ones from the cache, the
        // step's new ones rotated from the projections (and written to the cache)
        for (int e = tid; e < (t1 - t0) * (hd / 2); e += kAttnThreads) {
            const int tt = e / (hd / 2), i = e % (hd / 2), t = t0 + tt;
            float k0, k1, v0, v1;
            if (t < pos) {
                const float *kr = p.kc + ((size_t)t * p.kvh + j) * hd;
                const float *vr = p.vc + ((size_t)t * p.kvh + j) * hd;
                k0 = kr[i];
                k1 = kr[i + hd / 2];
                v0 = vr[i];
                v1 = vr[i + hd / 2];
            } else {
                const int m = t - pos;
                const float *kr = p.k + (size_t)m * p.ldkv + (size_t)j * hd;
                const float *vr = p.v + (size_t)m * p.ldkv + (size_t)j * hd;
                float c, s;
                rope_cs(i, hd, p.theta, t, c, s);
                const float a = kr[i], b = kr[i + hd / 2];
                k0 = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
                k1 = __fadd_rn(__fmul_rn(a, s), __fmul_rn(b, c));
                v0 = vr[i];
                v1 = vr[i + hd / 2];
                float *kw = p.kc + ((size_t)t * p.kvh + j) * hd;
                float *vw = p.vc + ((size_t)t * p.kvh + j) * hd;
                kw[i] = k0;
                kw[i + hd / 2] = k1;
                vw[i] = v0;
                vw[i + hd / 2] = v1;
            }
            ks[tt * ldk + i] = k0;
            ks[tt * ldk + i + hd / 2] = k1;
            vs[tt * hd + i] = v0;
            vs[tt * hd + i + hd / 2] = v1;
        }
        __syncthreads();
        // scores and the partial softmax: warp w takes queries w, w + 8, ...;
        // lane l takes positions t0 + l and t0 + l + 32
        for (int qi = warp; qi < NQ; qi += kAttnThreads / 32) {
            const int m = qi % p.M;
            const int lim = pos + m;  // last position this query sees
            float sc[kAttnTc / 32];
            float mx = -INFINITY;
#pragma unroll
            for (int r = 0; r < kAttnTc / 32; ++r) {
                const int tt = lane + 32 * r, t = t0 + tt;
                float d = 0.0f;
                if (t < t1 && t <= lim) {
                    const float *qr = qs + qi * hd, *kr = ks + tt * ldk;
#pragma unroll 8
                    for (int x = 0; x < hd; ++x) d = fmaf(qr[x], kr[x], d);
                    d = __fmul_rn(d, p.scale);
                } else {
                    d = -INFINITY;
                }
                sc[r] = d;
                mx = fmaxf(mx, d);
            }
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
            float l = 0.0f;
#pragma unroll
            for (int r = 0; r < kAttnTc / 32; ++r) {
                const float e = sc[r] == -INFINITY ? 0.0f : expf(sc[r] - mx);
                ps[qi * kAttnTc + lane + 32 * r] = e;
                l += e;
            }
#pragma unroll
            for (int off = 16; off > 0; off >>= 1) l += __shfl_xor_sync(0xffffffffu, l, off);
            __syncwarp();
            float *pr = p.part + (((size_t)j * p.nsplit + sp) * kAttnMaxQ + qi) * (hd + 2);
            for (int x = lane; x < hd; x += 32) {
                float o = 0.0f;
                for (int tt = 0; tt < t1 - t0; ++tt) o = fmaf(ps[qi * kAttnTc + tt], vs[tt * hd + x], o);
                pr[2 + x] = o;
            }
            if (lane == 0) {
                pr[0] = mx;
                pr[1] = l;
            }
        }
    }
    // the last CTA of this kv head combines every split in split order (every
    // thread's partials are made visible at device scope before the arrival)
    __threadfence();
    __syncthreads();
    if (tid == 0) s_last = atomicAdd(&p.ctr[j], 1u) == (unsigned)(gridDim.y - 1);
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    const int nact = (tmax + kAttnTc - 1) / kAttnTc;  // splits that hold positions
    for (int qi = warp; qi < NQ; qi += kAttnThreads / 32) {
        const int g = qi / p.M, m = qi % p.M;
        float mx = -INFINITY;
        for (int s2 = 0; s2 < nact; ++s2) {
            const float *pr = p.part + (((size_t)j * p.nsplit + s2) * kAttnMaxQ + qi) * (hd + 2);
            mx = fmaxf(mx, __ldcg(pr));
        }
        float L = 0.0f;
        for (int s2 = 0; s2 < nact; ++s2) {
            const float *pr = p.part + (((size_t)j * p.nsplit + s2) * kAttnMaxQ + qi) * (hd + 2);
            const float ms = __ldcg(pr);
            if (ms != -INFINITY) L = fmaf(expf(ms - mx), __ldcg(pr + 1), L);
        }
        const float invL = __fdiv_rn(1.0f, L);
        const int head = j * G + g;
        const float *gate = p.q + (size_t)m * p.ldq + (size_t)head * qstride + hd;
        for (int x = lane; x < hd; x += 32) {
            float o = 0.0f;
            for (int s2 = 0; s2 < nact; ++s2) {
                const float *pr = p.part + (((size_t)j * p.nsplit + s2) * kAttnMaxQ + qi) * (hd + 2);
                const float ms = __ldcg(pr);
                if (ms != -INFINITY) o = fmaf(expf(ms - mx), __ldcg(pr + 2 + x), o);
            }
            o = __fmul_rn(o, invL);
            if (p.gated) o = __fmul_rn(o, __fdiv_rn(1.0f, __fadd_rn(1.0f, exp_rn(-gate[x]))));
            p.out[(size_t)m * p.ldo + (size_t)head * hd + x] = o;
        }
    }
    if (tid == 0) p.ctr[j] = 0u;  // clean for the next launch
}

struct DeltaParams {
    const float *qkv;  // rows [M][ldqkv]: q (H x dk), k (H x dk), v (H x dv) channels
    int ldqkv;
    const float *convw;  // [C][4] conv taps per channel (tap k weighs the input k positions back)
    float *ring;         // [kRingSlots][C] inputs of earlier positions (slot = position % kRingSlots)
    float *state;        // [H][dk][dv]
    const float *decay;  // [H]
    const int *pos;
    int M, H, dk, dv, C;
    float *out;  // rows [M][ldo]: H x dv
    int ldo;
};

constexpr int kDeltaThreads = 256;
constexpr int kDeltaSlab = 32;  // value columns per CTA (one per lane)

// conv1d output of channel c at position t (src/ssm.zig:26-41): the sum over
// taps k = 0..3, in that order, of input(t - k) * w[c][k]; input(tau) is the
// step's row tau - pos for tau >= pos, the ring for earlier positions, 0
// before the sequence.
__device__ __forceinline__ float conv_at(const DeltaParams &p, int c, int t, int pos) {
    float sum = 0.0f;
#pragma unroll
    for (int k = 0; k < kConvWidth; ++k) {
        const int tau = t - k;
        float x = 0.0f;
        if (tau >= pos)
            x = p.qkv[(size_t)(tau - pos) * p.ldqkv + c];
        else if (tau >= 0)
            x = p.ring[(size_t)(tau % kRingSlots) * p.C + c];
        sum = __fadd_rn(sum, __fmul_rn(x, p.convw[(size_t)c * kConvWidth + k]));
    }
    return sum;
}

__global__ void __launch_bounds__(kDeltaThreads) chpe_deltanet_kernel(const DeltaParams p) {
    __shared__ float qs[128], ks[128], vs[kDeltaSlab];
    __shared__ float red[kDeltaThreads / 32][kDeltaSlab];
    pdl_begin();
    const int h = blockIdx.x, slab = blockIdx.y;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int dk = p.dk, rows_per_warp = dk / (kDeltaThreads / 32);  // 16 for dk = 128
    const int col = slab * kDeltaSlab + lane;
    const int pos = *p.pos;
    const float alpha = p.decay[h];
    float S[16];
    float *st = p.state + (size_t)h * dk * p.dv;
#pragma unroll
    for (int r = 0; r < 16; ++r) S[r] = r < rows_per_warp ? st[(size_t)(warp * rows_per_warp + r) * p.dv + col] : 0.0f;
    const int cq = h * dk, ck = p.H * dk + h * dk, cv = 2 * p.H * dk + h * p.dv + slab * kDeltaSlab;
    for (int m = 0; m < p.M; ++m) {
        const int t = pos + m;
        if (tid < dk) qs[tid] = conv_at(p, cq + tid, t, pos);
        else if (tid < 2 * dk) ks[tid - dk] = conv_at(p, ck + tid - dk, t, pos);
        if (tid < kDeltaSlab) vs[tid] = conv_at(p, cv + tid, t, pos);
        __syncthreads();
        // S = alpha * S + k^T v, then this warp's part of y = q S (src/ssm.zig:70-98)
        const float vj = vs[lane];
        float y = 0.0f;
#pragma unroll
        for (int r = 0; r < 16; ++r) {
            if (r < rows_per_warp) {
                const int i = warp * rows_per_warp + r;
                S[r] = __fadd_rn(__fmul_rn(S[r], alpha), __fmul_rn(ks[i], vj));
                y = __fadd_rn(y, __fmul_rn(qs[i], S[r]));
            }
        }
        red[warp][lane] = y;
        __syncthreads();
        if (warp == 0) {
            float acc = 0.0f;
#pragma unroll
            for (int w = 0; w < kDeltaThreads / 32; ++w) acc = __fadd_rn(acc, red[w][lane]);
            p.out[(size_t)m * p.ldo + (size_t)h * p.dv + col] = acc;
        }
        __syncthreads();
    }
#pragma unroll
    for (int r = 0; r < 16; ++r)
        if (r < rows_per_warp) st[(size_t)(warp * rows_per_warp + r) * p.dv + col] = S[r];
    // the step's inputs enter the ring (positions pos .. pos + M - 1); each
    // channel is written by one CTA: q and k channels of head h by slab 0,
    // value channels by their slab
    for (int m = 0; m < p.M; ++m) {
        float *slot = p.ring + (size_t)((pos + m) % kRingSlots) * p.C;
        const float *row = p.qkv + (size_t)m * p.ldqkv;
        if (slab == 0 && tid < 2 * dk) {
            const int c = tid < dk ? cq + tid : ck + tid - dk;
            slot[c] = row[c];
        }
        if (tid < kDeltaSlab) slot[cv + tid] = row[cv + tid];
    }
}

__global__ void chpe_pos_advance_kernel(int *pos, int M) {
    pdl_begin();
    if (threadIdx.x == 0 && blockIdx.x == 0) *pos += M;
}

size_t attn_smem_bytes(int NQ, int hd) {
    return ((size_t)NQ * hd + (size_t)kAttnTc * (hd + 1) + (size_t)kAttnTc * hd + (size_t)NQ * kAttnTc) * sizeof(float);
}

}  // namespace chpe

using namespace chpe;

int *chpe_ctx_error_word(chpe_ctx *ctx);
int chpe_ctx_scratch(chpe_ctx *ctx, int slot, size_t bytes, void **out);

extern "C" int chpe_attn_decode_dev(chpe_ctx *ctx, const float *q, int ldq, const float *k, const float *v, int ldkv,
                                    float *kcache, float *vcache, const int *pos, int M, int q_heads, int kv_heads,
                                    int head_dim, int max_seq, float rope_theta, int gated, float *out, int ldo,
                                    void *stream) {
    if (!ctx || !q || !k || !v || !kcache || !vcache || !pos || !out) return CHPE_EINVAL;
    if (M < 1 || M > kMaxTokens || kv_heads < 1 || q_heads < kv_heads || q_heads % kv_heads) return CHPE_EINVAL;
    if (head_dim < 2 || head_dim % 2 || head_dim > 256 || max_seq < M) return CHPE_EINVAL;
    const int G = q_heads / kv_heads, NQ = G * M;
    if (NQ > kAttnMaxQ) return CHPE_ENOTSUP;
    const size_t smem = attn_smem_bytes(NQ, head_dim);
    if (smem > 220 * 1024) return CHPE_ENOTSUP;
    AttnParams p;
    p.q = q;
    p.k = k;
    p.v = v;
    p.ldq = ldq;
    p.ldkv = ldkv;
    p.kc = kcache;
    p.vc = vcache;
    p.pos = pos;
    p.M = M;
    p.qh = q_heads;
    p.kvh = kv_heads;
    p.hd = head_dim;
    p.max_seq = max_seq;
    p.gated = gated ? 1 : 0;
    p.theta = rope_theta;
    p.scale = 1.0f / sqrtf((float)head_dim);
    p.out = out;
    p.ldo = ldo;
    p.nsplit = (max_seq + kAttnTc - 1) / kAttnTc;
    const size_t part_bytes = (size_t)kv_heads * p.nsplit * kAttnMaxQ * (head_dim + 2) * sizeof(float);
    void *part = nullptr, *ctr = nullptr;
    int rc = chpe_ctx_scratch(ctx, 0, part_bytes, &part);
    if (rc) return rc;
    rc = chpe_ctx_scratch(ctx, 1, 64 * sizeof(unsigned), &ctr);  // zeroed when allocated; self-resetting
    if (rc) return rc;
    p.part = static_cast<float *>(part);
    p.ctr = static_cast<unsigned *>(ctr);
    p.err = chpe_ctx_error_word(ctx);
    if (kv_heads > 64) return CHPE_ENOTSUP;
    static KernelDeviceState kstate;
    cudaError_t e = kernel_prepare(kstate, chpe_attn_decode_kernel, kAttnThreads, 220 * 1024, smem, nullptr);
    if (e == cudaSuccess)
        e = launch_pdl(chpe_attn_decode_kernel, dim3(kv_heads, p.nsplit), dim3(kAttnThreads), smem,
                       static_cast<cudaStream_t>(stream), p);
    return e == cudaSuccess ? CHPE_OK : CHPE_ECUDA;
}

extern "C" int chpe_deltanet_step_dev(chpe_ctx *ctx, const float *qkv, int ldqkv, const float *conv_w, float *ring,
                                      float *state, const float *decay, const int *pos, int M, int heads, int key_dim,
                                      int value_dim, float *out, int ldo, void *stream) {
    if (!ctx || !qkv || !conv_w || !ring || !state || !decay || !pos || !out) return CHPE_EINVAL;
    if (M < 1 || M > kRingSlots - (kConvWidth - 1) || heads < 1) return CHPE_EINVAL;
    if (key_dim != 128 || value_dim % kDeltaSlab || value_dim < kDeltaSlab) return CHPE_ENOTSUP;
    DeltaParams p;
    p.qkv = qkv;
    p.ldqkv = ldqkv;
    p.convw = conv_w;
    p.ring = ring;
    p.state = state;
    p.decay = decay;
    p.pos = pos;
    p.M = M;
    p.H = heads;
    p.dk = key_dim;
    p.dv = value_dim;
    p.C = heads * (2 * key_dim + value_dim);
    p.out = out;
    p.ldo = ldo;
    cudaError_t e = launch_pdl(chpe_deltanet_kernel, dim3(heads, value_dim / kDeltaSlab), dim3(kDeltaThreads), 0,
                               static_cast<cudaStream_t>(stream), p);
    return e == cudaSuccess ? CHPE_OK : CHPE_ECUDA;
}

extern "C" int chpe_pos_advance_dev(chpe_ctx *ctx, int *pos, int M, void *stream) {
    if (!ctx || !pos || M < 0) return CHPE_EINVAL;
    cudaError_t e = launch_pdl(chpe_pos_advance_kernel, dim3(1), dim3(32), 0, static_cast<cudaStream_t>(stream), pos, M);
    return e == cudaSuccess ? CHPE_OK : CHPE_ECUDA;
}
