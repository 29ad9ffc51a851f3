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
#include <unordered_map>

#include "../../include/chpe_b200.h"
#include "common.cuh"
#include "internal.h"
#include "xsrc.cuh"

namespace chpe {

constexpr int kAttnTc = 32;        // positions per attention CTA (one per lane)
constexpr int kAttnThreads = 256;
constexpr int kAttnMaxQ = 64;      // queries per CTA: group (q heads per kv head) x rows
constexpr int kRingSlots = 16;     // conv ring positions per channel (>= rows + 3)
constexpr int kConvWidth = 4;
constexpr int kErrCacheFull = 41;  // a step past the KV cache's max_seq positions
constexpr int kAttnMaxSplits = 1024;  // max_seq <= 32 K positions

// RoPE factors of pair i of a head_dim-wide head at position p, as the
// reference computes them (f32: e = 2i / head_dim, freq = 1 / theta^e,
// angle = p * freq) with pow, cos and sin taken in double and rounded to
// float -- the oracle does the same, so both get the same bits.  They are
// tabulated once per (theta, head_dim, max_seq): cs[p][i] = (cos, sin).
__global__ void chpe_rope_table_kernel(float theta, int head_dim, int max_seq, float2 *__restrict__ cs) {
    const int h2 = head_dim / 2;
    for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < max_seq * h2; e += gridDim.x * blockDim.x) {
        const int p = e / h2, i = e % h2;
        const float ex = __fdiv_rn(2.0f * (float)i, (float)head_dim);
        const float freq = __fdiv_rn(1.0f, (float)pow((double)theta, (double)ex));
        const float ang = __fmul_rn((float)p, freq);
        cs[e] = make_float2((float)cos((double)ang), (float)sin((double)ang));
    }
}

struct AttnParams {
    const float *q;  // rows [M][ldq]: per q head, head_dim query values (then head_dim gate values when gated)
    const float *k, *v;  // rows [M][ldkv]: kv_heads x head_dim
    int ldq, ldkv;
    float *kc, *vc;  // this layer's cache [max_seq][kv_heads][head_dim]
    const float2 *rope;  // (cos, sin) [max_seq][head_dim / 2]
    const int *pos;
    int M, qh, kvh, hd, max_seq, gated;
    float scale;
    float *out;  // rows [M][ldo]: q_heads x head_dim
    int ldo;
    float *part;  // partials [kvh][nsplit][kAttnMaxQ][hd + 2]: (max, sum, weighted values)
    int nsplit;
    int *err;
};

// Scores and partial softmax of one kv head over one split of kAttnTc
// positions, for one group of up to 8 * QPW of its queries (G q heads x M
// rows, query qi = g * M + m; grid: kv head x split x query group).  Lane l of
// every warp takes position t0 + l; warp w takes queries w, w + 8, ... of the
// group, so each key and value element is loaded once for all of a warp's
// queries; NCOL = head_dim / 32 columns per lane in the weighted value sum.
template <int QPW, int NCOL>
__global__ void __launch_bounds__(kAttnThreads) chpe_attn_partial_kernel(const AttnParams p) {
    extern __shared__ __align__(16) float sm[];
    pdl_begin();
    constexpr int QG = 8 * QPW;  // queries per CTA
    const int j = blockIdx.x;    // kv head
    const int sp = blockIdx.y;
    const int q0 = blockIdx.z * QG;
    const int hd = p.hd, h2 = hd / 2, G = p.qh / p.kvh, NQ = G * p.M;
    const int nqc = min(QG, NQ - q0);  // queries of this CTA
    const int pos = *p.pos;
    const int tmax = pos + p.M;  // positions after this step
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (pos < 0 || tmax > p.max_seq) {  // the cache is full: record it, touch nothing (every CTA returns)
        if (j == 0 && sp == 0 && blockIdx.z == 0 && tid == 0) atomicExch(p.err, kErrCacheFull);
        return;
    }
    const int t0 = sp * kAttnTc, t1 = min(t0 + kAttnTc, tmax);
    if (t0 >= t1 || nqc <= 0) return;  // past the sequence
    const int ldk = hd + 1;  // padded rows: lanes read different positions without bank conflicts
    float *qs = sm;                  // [QG][hd]
    float *vs = qs + QG * hd;        // [kAttnTc][hd] (16-byte aligned rows)
    float *ks = vs + kAttnTc * hd;   // [kAttnTc][hd + 1]
    float *ps = ks + kAttnTc * ldk;  // [QG][kAttnTc] probabilities
    const int qstride = p.gated ? 2 * hd : hd;
    // rotated queries of the group
    for (int e = tid; e < nqc * h2; e += kAttnThreads) {
        const int ql = e / h2, i = e % h2, qi = q0 + ql;
        const int g = qi / p.M, m = qi % p.M;
        const float *src = p.q + (size_t)m * p.ldq + (size_t)(j * G + g) * qstride;
        const float2 cs = p.rope[(size_t)(pos + m) * h2 + i];
        const float v0 = src[i], v1 = src[i + h2];
        qs[ql * hd + i] = __fsub_rn(__fmul_rn(v0, cs.x), __fmul_rn(v1, cs.y));
        qs[ql * hd + i + h2] = __fadd_rn(__fmul_rn(v0, cs.y), __fmul_rn(v1, cs.x));
    }
    // keys and values of cached positions t0 .. min(t1, pos)-1: 16-byte
    // granules, all loads in flight before the first store
    const int tc = min(t1, pos);
    const int g4 = hd / 4;
    const int ngran = (tc > t0 ? tc - t0 : 0) * g4;
    constexpr int U = kAttnTc * 64 / kAttnThreads;  // granules per thread (head_dim <= 256)
    {
        float4 kr[U], vr[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int gi = u * kAttnThreads + tid;
            if (gi < ngran) {
                const int t = t0 + gi / g4, x4 = gi % g4;
                const size_t off = ((size_t)t * p.kvh + j) * hd + 4 * x4;
                kr[u] = __ldg(reinterpret_cast<const float4 *>(p.kc + off));
                vr[u] = __ldg(reinterpret_cast<const float4 *>(p.vc + off));
            }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
            const int gi = u * kAttnThreads + tid;
            if (gi < ngran) {
                const int tt = gi / g4, x = 4 * (gi % g4);
                float *kd = ks + tt * ldk + x;
                kd[0] = kr[u].x;
                kd[1] = kr[u].y;
                kd[2] = kr[u].z;
                kd[3] = kr[u].w;
                *reinterpret_cast<float4 *>(vs + tt * hd + x) = vr[u];
            }
        }
    }
    // the step's new positions in this split: rotated from the projections;
    // the first query group's CTA writes them to the cache
    for (int e = tid; e < (t1 > pos ? t1 - max(t0, pos) : 0) * h2; e += kAttnThreads) {
        const int t = max(t0, pos) + e / h2, i = e % h2, tt = t - t0, m = t - pos;
        const float *kr = p.k + (size_t)m * p.ldkv + (size_t)j * hd;
        const float *vr = p.v + (size_t)m * p.ldkv + (size_t)j * hd;
        const float2 cs = p.rope[(size_t)t * h2 + i];
        const float a = kr[i], b = kr[i + h2];
        const float k0 = __fsub_rn(__fmul_rn(a, cs.x), __fmul_rn(b, cs.y));
        const float k1 = __fadd_rn(__fmul_rn(a, cs.y), __fmul_rn(b, cs.x));
        const float v0 = vr[i], v1 = vr[i + h2];
        if (blockIdx.z == 0) {
            float *kw = p.kc + ((size_t)t * p.kvh + j) * hd;
            float *vw = p.vc + ((size_t)t * p.kvh + j) * hd;
            kw[i] = k0;
            kw[i + h2] = k1;
            vw[i] = v0;
            vw[i + h2] = v1;
        }
        ks[tt * ldk + i] = k0;
        ks[tt * ldk + i + h2] = k1;
        vs[tt * hd + i] = v0;
        vs[tt * hd + i + h2] = v1;
    }
    __syncthreads();
    const int nq = (nqc - warp + 7) / 8;  // queries of this warp
    if (nq <= 0) return;
    const int n = t1 - t0;
    float sc[QPW];
#pragma unroll
    for (int a = 0; a < QPW; ++a) sc[a] = 0.0f;
    const float *kr = ks + lane * ldk;
#pragma unroll 4
    for (int x = 0; x < hd; ++x) {
        const float kx = kr[x];
#pragma unroll
        for (int a = 0; a < QPW; ++a) sc[a] = fmaf(qs[(warp + 8 * a) * hd + x], kx, sc[a]);
    }
    float mxs[QPW], ls[QPW];
#pragma unroll
    for (int a = 0; a < QPW; ++a) {
        const int ql = warp + 8 * a, lim = pos + (q0 + ql) % p.M;  // last position this query sees
        float v = (a < nq && lane < n && t0 + lane <= lim) ? __fmul_rn(sc[a], p.scale) : -INFINITY;
        float mx = v;
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
        const float e = v == -INFINITY ? 0.0f : expf(v - mx);
        float l = e;
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) l += __shfl_xor_sync(0xffffffffu, l, off);
        if (a < nq) ps[ql * kAttnTc + lane] = e;
        mxs[a] = mx;
        ls[a] = l;
    }
    __syncwarp();
    float o[QPW][NCOL];
#pragma unroll
    for (int a = 0; a < QPW; ++a)
#pragma unroll
        for (int c = 0; c < NCOL; ++c) o[a][c] = 0.0f;
    for (int tt = 0; tt < n; ++tt) {
        float vv[NCOL];
#pragma unroll
        for (int c = 0; c < NCOL; ++c) vv[c] = vs[tt * hd + lane + 32 * c];
#pragma unroll
        for (int a = 0; a < QPW; ++a) {
            const float pw = a < nq ? ps[(warp + 8 * a) * kAttnTc + tt] : 0.0f;
#pragma unroll
            for (int c = 0; c < NCOL; ++c) o[a][c] = fmaf(pw, vv[c], o[a][c]);
        }
    }
#pragma unroll
    for (int a = 0; a < QPW; ++a) {
        if (a >= nq) continue;
        const int qi = q0 + warp + 8 * a;
        float *pr = p.part + (((size_t)j * p.nsplit + sp) * kAttnMaxQ + qi) * (hd + 2);
#pragma unroll
        for (int c = 0; c < NCOL; ++c) pr[2 + lane + 32 * c] = o[a][c];
        if (lane == 0) {
            pr[0] = mxs[a];
            pr[1] = ls[a];
        }
    }
}

// Combines the splits of one query head and row (grid q_heads x M, head_dim
// threads): out = sum_s e^(m_s - M) o_s / sum_s e^(m_s - M) l_s over the
// splits in order, times sigmoid(gate) when gated.
__global__ void __launch_bounds__(256) chpe_attn_combine_kernel(const AttnParams p) {
    __shared__ float wts[kAttnMaxSplits];
    __shared__ float s_inv;
    pdl_begin();
    const int head = blockIdx.x, m = blockIdx.y, x = threadIdx.x;
    const int pos = *p.pos;
    const int tmax = pos + p.M;
    if (pos < 0 || tmax > p.max_seq) return;  // recorded by the partial kernel
    const int hd = p.hd, G = p.qh / p.kvh, j = head / G, g = head % G, qi = g * p.M + m;
    const int nact = (tmax + kAttnTc - 1) / kAttnTc;
    const float *pbase = p.part + ((size_t)j * p.nsplit * kAttnMaxQ + qi) * (hd + 2);
    const size_t sstride = (size_t)kAttnMaxQ * (hd + 2);
    if (threadIdx.x < 32) {
        // split maxima and sums: lane s reads split s (nact <= kAttnMaxSplits)
        float mx = -INFINITY;
        for (int s2 = threadIdx.x; s2 < nact; s2 += 32) mx = fmaxf(mx, __ldcg(pbase + s2 * sstride));
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
        for (int s2 = threadIdx.x; s2 < nact; s2 += 32) {
            const float ms = __ldcg(pbase + s2 * sstride);
            wts[s2] = ms == -INFINITY ? 0.0f : expf(ms - mx);
        }
        __syncwarp();
        if (threadIdx.x == 0) {
            float L = 0.0f;
            for (int s2 = 0; s2 < nact; ++s2) L = fmaf(wts[s2], __ldcg(pbase + s2 * sstride + 1), L);
            s_inv = __fdiv_rn(1.0f, L);
        }
    }
    __syncthreads();
    if (x >= hd) return;
    float o = 0.0f;
    for (int s2 = 0; s2 < nact; ++s2) o = fmaf(wts[s2], __ldcg(pbase + s2 * sstride + 2 + x), o);
    o = __fmul_rn(o, s_inv);
    if (p.gated) {
        const float gt = p.q[(size_t)m * p.ldq + (size_t)head * 2 * hd + hd + x];
        o = __fmul_rn(o, __fdiv_rn(1.0f, __fadd_rn(1.0f, exp_rn(-gt))));
    }
    p.out[(size_t)m * p.ldo + (size_t)head * hd + x] = o;
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
constexpr int kMaxDeltaRows = 8;  // rows per call

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
    __shared__ float qs[kMaxDeltaRows][128], ks[kMaxDeltaRows][128], vs[kMaxDeltaRows][kDeltaSlab];
    __shared__ float red[kMaxDeltaRows][kDeltaThreads / 32][kDeltaSlab];
    pdl_begin();
    const int h = blockIdx.x, slab = blockIdx.y;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int dk = p.dk, rows_per_warp = dk / (kDeltaThreads / 32);  // 16 for dk = 128
    const int col = slab * kDeltaSlab + lane;
    const int pos = *p.pos;
    const int M = p.M;
    const float alpha = p.decay[h];
    const int cq = h * dk, ck = p.H * dk + h * dk, cv = 2 * p.H * dk + h * p.dv + slab * kDeltaSlab;
    // conv1d outputs of every row first (they depend on the inputs only): all loads in flight at once
    for (int e = tid; e < M * (2 * dk + kDeltaSlab); e += kDeltaThreads) {
        const int m = e / (2 * dk + kDeltaSlab), c = e % (2 * dk + kDeltaSlab);
        if (c < dk) qs[m][c] = conv_at(p, cq + c, pos + m, pos);
        else if (c < 2 * dk) ks[m][c - dk] = conv_at(p, ck + c - dk, pos + m, pos);
        else vs[m][c - 2 * dk] = conv_at(p, cv + c - 2 * dk, pos + m, pos);
    }
    float S[16];
    float *st = p.state + (size_t)h * dk * p.dv;
#pragma unroll
    for (int r = 0; r < 16; ++r) S[r] = r < rows_per_warp ? st[(size_t)(warp * rows_per_warp + r) * p.dv + col] : 0.0f;
    __syncthreads();
    // rows in order: S = alpha * S + k^T v, then this warp's part of y = q S (src/ssm.zig:70-98)
    for (int m = 0; m < M; ++m) {
        const float vj = vs[m][lane];
        float y = 0.0f;
#pragma unroll
        for (int r = 0; r < 16; ++r) {
            if (r < rows_per_warp) {
                const int i = warp * rows_per_warp + r;
                S[r] = __fadd_rn(__fmul_rn(S[r], alpha), __fmul_rn(ks[m][i], vj));
                y = __fadd_rn(y, __fmul_rn(qs[m][i], S[r]));
            }
        }
        red[m][warp][lane] = y;
    }
#pragma unroll
    for (int r = 0; r < 16; ++r)
        if (r < rows_per_warp) st[(size_t)(warp * rows_per_warp + r) * p.dv + col] = S[r];
    __syncthreads();
    // warp m sums row m's warp partials in warp order
    for (int m = warp; m < M; m += kDeltaThreads / 32) {
        float acc = 0.0f;
#pragma unroll
        for (int w = 0; w < kDeltaThreads / 32; ++w) acc = __fadd_rn(acc, red[m][w][lane]);
        p.out[(size_t)m * p.ldo + (size_t)h * p.dv + col] = acc;
    }
    // the step's inputs enter the ring (positions pos .. pos + M - 1); each
    // channel is written by one CTA: q and k channels of head h by slab 0,
    // value channels by their slab
    for (int e = tid; e < M * (2 * dk + kDeltaSlab); e += kDeltaThreads) {
        const int m = e / (2 * dk + kDeltaSlab), c = e % (2 * dk + kDeltaSlab);
        float *slot = p.ring + (size_t)((pos + m) % kRingSlots) * p.C;
        const float *row = p.qkv + (size_t)m * p.ldqkv;
        int ch;
        if (c < 2 * dk) {
            if (slab != 0) continue;
            ch = c < dk ? cq + c : ck + c - dk;
        } else {
            ch = cv + c - 2 * dk;
        }
        slot[ch] = row[ch];
    }
}

__global__ void chpe_pos_advance_kernel(int *pos, int M) {
    pdl_begin();
    if (threadIdx.x == 0 && blockIdx.x == 0) *pos += M;
}

size_t attn_smem_bytes(int QG, int hd) {
    return ((size_t)QG * hd + (size_t)kAttnTc * hd + (size_t)kAttnTc * (hd + 1) + (size_t)QG * kAttnTc) *
           sizeof(float);
}

// Queries per warp of the partial kernel for a group of NQ queries: the
// smallest of 1, 2, 4 with 8 * QPW >= NQ (groups of 32 above).
static int attn_qpw(int NQ) { return NQ <= 8 ? 1 : NQ <= 16 ? 2 : 4; }

template <int QPW, int NCOL>
static cudaError_t launch_attn_partial(const AttnParams &p, int nqg, cudaStream_t st) {
    static KernelDeviceState kstate;
    const size_t smem = attn_smem_bytes(8 * QPW, p.hd);
    auto kern = chpe_attn_partial_kernel<QPW, NCOL>;
    cudaError_t e = kernel_prepare(kstate, kern, kAttnThreads, 220 * 1024, smem, nullptr);
    if (e != cudaSuccess) return e;
    return launch_pdl(kern, dim3(p.kvh, p.nsplit, nqg), dim3(kAttnThreads), smem, st, p);
}

}  // namespace chpe

using namespace chpe;

int *chpe_ctx_error_word(chpe_ctx *ctx);
int chpe_ctx_scratch(chpe_ctx *ctx, int slot, size_t bytes, void **out);
unsigned chpe_ctx_scratch_generation(chpe_ctx *ctx, int slot);
unsigned chpe_ctx_scratch_seen(chpe_ctx *ctx, int slot);
void chpe_ctx_scratch_mark_seen(chpe_ctx *ctx, int slot);

// RoPE table of (theta, head_dim, max_seq) in the context's scratch slot 2
// (computed on first use: the first call must come before any stream capture).
static int rope_table(chpe_ctx *ctx, float theta, int head_dim, int max_seq, const float2 **out, cudaStream_t st) {
    struct Key {
        float theta;
        int hd, max_seq;
    };
    static thread_local std::unordered_map<chpe_ctx *, Key> keys;
    const size_t bytes = (size_t)max_seq * (head_dim / 2) * sizeof(float2);
    void *buf = nullptr;
    int rc = chpe_ctx_scratch(ctx, 2, bytes, &buf);
    if (rc) return rc;
    auto it = keys.find(ctx);
    if (it == keys.end() || it->second.theta != theta || it->second.hd != head_dim || it->second.max_seq < max_seq ||
        chpe_ctx_scratch_generation(ctx, 2) != chpe_ctx_scratch_seen(ctx, 2)) {
        note_launch();
        chpe_rope_table_kernel<<<256, 256, 0, st>>>(theta, head_dim, max_seq, static_cast<float2 *>(buf));
        if (cudaGetLastError() != cudaSuccess) return CHPE_ECUDA;
        if (cudaStreamSynchronize(st) != cudaSuccess) return CHPE_ECUDA;
        keys[ctx] = Key{theta, head_dim, max_seq};
        chpe_ctx_scratch_mark_seen(ctx, 2);
    }
    *out = static_cast<const float2 *>(buf);
    return CHPE_OK;
}

extern "C" int chpe_attn_decode_dev(chpe_ctx *ctx, const float *q, int ldq, const float *k, const float *v, int ldkv,
                                    float *kcache, float *vcache, const int *pos, int M, int q_heads, int kv_heads,
                                    int head_dim, int max_seq, float rope_theta, int gated, float *out, int ldo,
                                    void *stream) {
    if (!ctx || !q || !k || !v || !kcache || !vcache || !pos || !out) return CHPE_EINVAL;
    if (M < 1 || M > kMaxTokens || kv_heads < 1 || q_heads < kv_heads || q_heads % kv_heads) return CHPE_EINVAL;
    if (head_dim < 2 || head_dim % 2 || head_dim > 256 || max_seq < M) return CHPE_EINVAL;
    const int G = q_heads / kv_heads, NQ = G * M;
    if (NQ > kAttnMaxQ) return CHPE_ENOTSUP;
    if (head_dim % 32) return CHPE_ENOTSUP;  // whole warps of columns (head_dim 32 .. 256)
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
    p.scale = 1.0f / sqrtf((float)head_dim);
    p.out = out;
    p.ldo = ldo;
    p.nsplit = (max_seq + kAttnTc - 1) / kAttnTc;
    if (p.nsplit > kAttnMaxSplits) return CHPE_ENOTSUP;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const size_t part_bytes = (size_t)kv_heads * p.nsplit * kAttnMaxQ * (head_dim + 2) * sizeof(float);
    void *part = nullptr;
    int rc = chpe_ctx_scratch(ctx, 0, part_bytes, &part);
    if (rc) return rc;
    if ((rc = rope_table(ctx, rope_theta, head_dim, max_seq, &p.rope, st))) return rc;
    p.part = static_cast<float *>(part);
    p.err = chpe_ctx_error_word(ctx);
    const int qpw = attn_qpw(NQ), nqg = (NQ + 8 * qpw - 1) / (8 * qpw), ncol = head_dim / 32;
    cudaError_t e;
#define CHPE_ATTN_NCOL(QPW)                                                                            \
    switch (ncol) {                                                                                    \
    case 1: e = launch_attn_partial<QPW, 1>(p, nqg, st); break;                                        \
    case 2: e = launch_attn_partial<QPW, 2>(p, nqg, st); break;                                        \
    case 4: e = launch_attn_partial<QPW, 4>(p, nqg, st); break;                                        \
    case 8: e = launch_attn_partial<QPW, 8>(p, nqg, st); break;                                        \
    default: return CHPE_ENOTSUP;                                                                      \
    }
    if (qpw == 1) {
        CHPE_ATTN_NCOL(1)
    } else if (qpw == 2) {
        CHPE_ATTN_NCOL(2)
    } else {
        CHPE_ATTN_NCOL(4)
    }
#undef CHPE_ATTN_NCOL
    if (e == cudaSuccess)
        e = launch_pdl(chpe_attn_combine_kernel, dim3(q_heads, M), dim3(head_dim < 32 ? 32 : head_dim), 0, st, p);
    return e == cudaSuccess ? CHPE_OK : CHPE_ECUDA;
}

extern "C" int chpe_deltanet_step_dev(chpe_ctx *ctx, const float *qkv, int ldqkv, const float *conv_w, float *ring,
                                      float *state, const float *decay, const int *pos, int M, int heads, int key_dim,
                                      int value_dim, float *out, int ldo, void *stream) {
    if (!ctx || !qkv || !conv_w || !ring || !state || !decay || !pos || !out) return CHPE_EINVAL;
    if (M < 1 || M > kMaxDeltaRows || heads < 1) return CHPE_EINVAL;
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
