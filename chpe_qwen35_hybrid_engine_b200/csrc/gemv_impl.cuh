// gemv_impl.cuh -- decode/verify GEMV kernel template for M = 1..8 activation
// rows over quantized weights in the strip layout (layout.h).  Instantiated per
// code width in gemv_b8.cu / gemv_b4.cu / gemv_b2.cu / gemv_s8.cu; planned and
// dispatched in gemv.cu.
//
// Persistent, warp-specialised kernel.  A CTA (8 MMA warps, 1 producer warp,
// 1 epilogue warp) is bound to one K-slice for its lifetime: its activation
// fragments are bulk-copied into shared memory once.  The slice's work is cut
// into units (strip groups, whole or in chunks of blocks; see unit_of).
// Every CTA takes its first units statically, so it can start fetching
// weights before the upstream kernel has finished, and the rest from a
// per-slice atomic work counter, so CTAs that stream faster take more units
// and all of them finish within about one unit of each other.  The producer
// warp streams each unit -- per strip and stage one block, 4 KiB of codes plus
// the block's group metadata, in one 1-D bulk copy (TMA engine, mbarrier
// completion, L2 evict-first) -- through a 3-stage shared-memory ring.  A
// strip group is four 16-row strips, or for the fused gate/up SwiGLU the same
// two strips of the gate and of the up matrix.
//
// Each MMA warp takes one chunk of every block, turns codes into fp16 MMA
// operands in registers with one LOP3 / PRMT per pair (the code as an exact
// fp16 subnormal, code * 2^-24 -- or code * 2^-24 * 2^4m for codes read at a
// higher bit position, with 2^-4m pre-applied to that k-step's activations),
// issues m16n8k16 MMAs against the staged activation fragments, and folds the
// per-group scale / zero-point into fp32 register accumulators:
//     acc += s * D + (-z * s * 2^-24) * sum(x over the block),  y = 2^24 * acc.
// The int8 x int8 path (W8A8) feeds raw codes to m16n8k32 integer MMAs and
// keeps exact int32 sums.  At the end of a unit the MMA warps hand their
// accumulators to the epilogue warp (shared memory, fixed warp order).  A
// strip group that is one unit over its whole K is finished there; otherwise
// the unit's sum goes to the workspace slot of its chunk, and the CTA that
// brings the last chunk of the strip group (acquire-release arrival count)
// sums all slots in chunk order.  The sum of a chunk does not depend on which
// CTA computed it, so results are deterministic.
#pragma once
#include <algorithm>
#include <type_traits>

#include "common.cuh"
#include "internal.h"
#include "xsrc.cuh"

namespace chpe {

constexpr int kNW = 8;      // MMA warps per CTA (one chunk of each block)
constexpr int kStages = 3;  // ring depth (blocks per strip); 2 when a stream's stages carry activations
constexpr int kProducerWarp = kNW, kEpilogueWarp = kNW + 1;
constexpr int kThreads = (kNW + 2) * 32;
// activation fragments staged per CTA: small enough for two CTAs per SM at
// M <= 2 (2 x (74 KB ring + 28 KB + reduction buffers) <= 220 KB); with more
// rows the reduction buffers already limit a CTA to one SM, which then stages
// as much of K as fits (fewer K-slices, fewer partials)
constexpr int kXMaxBytes = 40 * 1024;
constexpr int kXMaxBytesWide = 100 * 1024;
constexpr size_t kTwoCtaBytes = 112 * 1024;  // dynamic shared memory of a CTA that shares its SM with another
constexpr int kSmemBudget = 220 * 1024;
constexpr size_t kSmemPerSm = 228 * 1024;  // shared memory of one SM, the CTAs' reserved 1 KB included
static_assert(kNW == kChunksPerBlock, "one block per stage, one chunk per warp");

// 16 bytes of zeros: the activation operand of MMA columns past the last row
constexpr size_t kZeroSlot = 496;

struct SmemLayout {
    size_t bar, tags, ring, xf, xs, red, info, xe, total;
    size_t stage;    // bytes of one ring stage
    size_t sx, sxs;  // streamed activations: offsets of a stage's fragments and block sums
    int nbuf;        // accumulator hand-off buffers (2 or 4)
};

// Hand-off of one finished unit from the MMA warps to the epilogue warp.
struct SegInfo {
    int sg;  // strip group, -1 = no more units
    int gc;  // chunk of the strip group's K
};

constexpr int kMaxRedBufs = 4;

__host__ __device__ inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Bytes of activation fragments per block of K (fp16 units of 16 bytes).
__host__ __device__ inline size_t xfrag_bytes_per_block(int layout, int bits, int M, bool xsplit) {
    const int steps = layout == kLayoutS8 ? 1 : (256 / bits) / 16;
    return (size_t)kChunksPerBlock * steps * M * 32 * (xsplit ? 2 : 1);
}

// Shared memory of one CTA.  Resident activations (xstream 0): the ring holds
// weights only and the CTA's K-slice of fragments and block sums sits in
// xf / xs.  Streamed activations (xstream 1): each ring stage carries, behind
// the block's weights, that block's fragments and block sums, and nothing is
// resident -- a CTA then covers all of K with no partial sums.
__host__ __device__ inline SmemLayout smem_layout(int layout, int bits, int bpk, int M, bool xsplit, int e_cols,
                                                  int block_bytes, int xstream = 0, int nstages = kStages) {
    SmemLayout L;
    // hand-off buffers: four at M <= 2 (the epilogue warp may spend an L2
    // round trip per unit without holding up the MMA warps), two above
    L.nbuf = M <= 2 ? kMaxRedBufs : 2;
    L.bar = 0;    // full[kStages], empty[kStages], xbar, rfull[kMaxRedBufs], rempty[kMaxRedBufs]
    L.tags = 256; // unit / block / flag tag per ring slot; 16 zero bytes at kZeroSlot
    size_t o = 512;
    static_assert((2 * kStages + 1 + 2 * kMaxRedBufs) * 8 <= 256 && 256 + 3 * kStages * 4 <= kZeroSlot,
                  "barrier / tag area");
    const size_t xblk = xfrag_bytes_per_block(layout, bits, M, xsplit);
    const size_t xsblk = layout == kLayoutF16 ? (size_t)kChunksPerBlock * ((256 / bits) / e_cols) * 32 : 0;
    L.sx = align_up((size_t)kSG * block_bytes, 128);
    L.sxs = align_up(L.sx + xblk, 128);
    L.stage = xstream ? align_up(L.sxs + xsblk, 128) : (size_t)kSG * block_bytes;
    L.ring = o;
    o += align_up((size_t)nstages * L.stage, 128);
    L.xf = o;
    if (!xstream) o = align_up(o + (size_t)bpk * xblk, 128);
    L.xs = o;
    if (!xstream && layout == kLayoutF16) o = align_up(o + (size_t)bpk * xsblk, 128);
    L.red = o;  // nbuf buffers of per-warp accumulators [warp][strip][16 rows][M]
    o += (size_t)L.nbuf * kNW * kSG * 16 * M * 4;
    L.info = o;
    o += kMaxRedBufs * sizeof(SegInfo);
    L.xe = o;  // row unscale factors of a fused fill [kMaxTokens]
    o += kMaxTokens * sizeof(float);
    L.total = align_up(o, 128);
    return L;
}

// Work units of one K-slice with nbk blocks.  Strip groups below n_whole are
// one unit each (all nbk blocks: long contiguous runs per strip, no partial
// sums within the slice); the others are cut into C chunks of bc blocks, so
// the last units handed out are short.  Unit u < n_whole is strip group u;
// unit n_whole + v is chunk v % C of strip group n_whole + v / C.  A CTA of the
// slice takes units j, j + Gk, ... (P of them) statically, then units
// P * Gk + g for the values g it draws from the slice's work counter, until
// one is past the last unit.  Each CTA draws exactly one such past-the-end
// value; the draw that returns the last value of the launch
// (grabs_total - 1) resets the counter for the next launch.
__host__ __device__ inline int unit_chunks(int nbk, int bc) { return (nbk + bc - 1) / bc; }

struct Unit {
    int sg, bs, be;  // strip group, blocks [bs, be) of the slice
    int gc, ctot;    // chunk index within the strip group's whole K, and its chunk count
};
// (32-bit arithmetic: a 64-bit division costs the producer a few hundred
// dependent instructions per unit, time in which no copy is issued)
__host__ __device__ inline Unit unit_of(int u, int nbk, int C, int ks, int n_ks, int n_whole, int bc, int cfull,
                                        int ctot_split) {
    if (u < n_whole) return Unit{u, 0, nbk, ks, n_ks};
    const unsigned v = (unsigned)(u - n_whole);
    const unsigned q = v / (unsigned)C;
    const int c = (int)(v - q * (unsigned)C);
    const int be = c * bc + bc < nbk ? c * bc + bc : nbk;
    return Unit{n_whole + (int)q, c * bc, be, ks * cfull + c, ctot_split};
}
__host__ __device__ inline int slice_units(int n_sg, int n_whole, int C) { return n_whole + (n_sg - n_whole) * C; }
// Static units per CTA: enough blocks to fill the ring before the first draw.
__host__ __device__ inline int static_units(int n_whole, int Gk, int nbk, int pref, int nstages) {
    return n_whole >= Gk ? (nstages + nbk - 1) / nbk : pref;
}
__host__ __device__ inline int grabs_total(int U, int pref, int Gk) { return (U > pref * Gk ? U - pref * Gk : 0) + Gk; }

// Codes become fp16 operands with the exponent field left at zero: the bit
// pattern `code` is the fp16 subnormal code * 2^-24, exact for every code
// (code < 1024).  One LOP3 (4/2-bit) or PRMT (8-bit) yields two operands and
// no subtraction is needed.  To avoid a shift per k-step, codes are masked in
// place in the low 8 bits of each half (w) or of each half of w >> 8: a code
// at bit 4 (4-bit) or bit 2m (2-bit) reads as code * 2^-24 * 16 (or * 4^m);
// the activations of that k-step were divided by the same power of two when
// the fragments were built (act_scale_shift), so every product is
// code * x * 2^-24.  The accumulator carries sum(code * x) only, so a small
// result next to a large zero-point term keeps fp32 precision.
template <int BITS>
__device__ __forceinline__ uint32_t unpack_f16(uint32_t w, uint32_t w8, int j) {
    if constexpr (BITS == 4) {
        const uint32_t src = j < 2 ? w : w8;
        return src & ((j & 1) ? 0x00F000F0u : 0x000F000Fu);
    } else if constexpr (BITS == 2) {
        const uint32_t src = j < 4 ? w : w8;
        return src & (0x00030003u << (2 * (j & 3)));
    } else {
        (void)w8;
        return __byte_perm(w, 0u, j == 0 ? 0x4140 : 0x4342);
    }
}

constexpr float kTwo24 = 16777216.0f;

constexpr float kTwoM24 = 1.0f / 16777216.0f;

// (scale, offset * 2^-24 per unit of x) of rows g and g+8 of one group; the
// block stores the two rows side by side, so one shared load fetches both.
// zc24 is the constant zero-point times -2^-24.  F32 metadata already holds
// the offset times 2^-24.
template <int META>
__device__ __forceinline__ void load_meta2(const uint8_t *gbase, int g, float zc24, float &s0, float &o0, float &s1,
                                           float &o1) {
    if constexpr (META == kMetaS16) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(gbase + g * 4));
        s0 = f.x;
        o0 = f.x * zc24;
        s1 = f.y;
        o1 = f.y * zc24;
    } else if constexpr (META == kMetaSZ16) {
        const uint2 v = *reinterpret_cast<const uint2 *>(gbase + g * 8);
        const float2 a = __half22float2(*reinterpret_cast<const __half2 *>(&v.x));
        const float2 b = __half22float2(*reinterpret_cast<const __half2 *>(&v.y));
        s0 = a.x;
        o0 = -(a.x * a.y) * kTwoM24;
        s1 = b.x;
        o1 = -(b.x * b.y) * kTwoM24;
    } else {
        const float4 f = *reinterpret_cast<const float4 *>(gbase + g * 16);
        s0 = f.x;
        o0 = f.y;
        s1 = f.z;
        o1 = f.w;
    }
}

// Source of strip i (0..kSG-1) of a strip group for the scale/zero constants:
// gate/up take strips 2sg, 2sg+1 of source 0 (gate, i = 0, 1) and of source 1
// (up, i = 2, 3); concatenated plain sources share one format.
template <int MODE>
__host__ __device__ __forceinline__ int source_of(int i) {
    return MODE == 1 ? (i >> 1) : 0;
}

// Strip i of strip group sg as (source, strip within that source's matrix),
// and whether it exists: plain GEMV -> strips 4(sg - sg0[r]) .. +3 of source r
// (the sources concatenated along N); gate/up -> as source_of.
struct StripRef {
    int r, strip;
    bool valid;
};
template <int MODE>
__device__ __forceinline__ StripRef strip_ref(const GemvParams &p, int sg, int i) {
    if (MODE == 1) {
        const int strip = 2 * sg + (i & 1);
        return StripRef{i >> 1, strip, strip < p.n_strips};
    }
    int r = 0;
#pragma unroll
    for (int k = 1; k < kMaxSrc; ++k) r += sg >= p.sg0[k];
    const int strip = kSG * (sg - p.sg0[r]) + i;
    return StripRef{r, strip, strip < p.nstr[r]};
}

// Output (or, for gate/up, the SwiGLU of the gate and up outputs) of entry
// q = (i * 16 + r) * M + tok of strip group sg from its summed accumulator(s):
// scales the integer (W8A8) sum, or the fp16 path's sum by 2^24 and by the
// row's unscale factor xe[tok] (the fill's power-of-two row scaling), adds
// the bias and the outlier columns, and writes or accumulates into y.
template <int LAYOUT, int MODE, typename Acc>
__device__ __forceinline__ void finalize_entry(const GemvParams &p, int sg, int q, Acc v, Acc v_up, const float *xe) {
    const int M = p.M;
    const int tok = q % M, ir = q / M, r = ir & 15, i = ir >> 4;
    const StripRef ref = strip_ref<MODE>(p, sg, i);
    const int row = ref.strip * kStripRows + r;
    if (!ref.valid || row >= (MODE == 1 ? p.N : p.rows[ref.r])) return;
    if (MODE == 0) {
        const GemvSrc &sr = p.src[ref.r];
        float out = LAYOUT == kLayoutS8 ? (float)v * (sr.scale * p.sx[tok]) : ((float)v * kTwo24) * xe[tok];
        if (sr.bias) out += sr.bias[row];
        if (sr.out_cols) {
            float os = 0.0f;
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                const int col = sr.out_cols[(size_t)row * 8 + c];
                if (col >= 0) os += __half2float(sr.out_w[(size_t)row * 8 + c]) * p.xrow[(size_t)tok * p.K + col];
            }
            out += os;
        }
        float *yp = p.ys[ref.r] + (size_t)tok * p.ldys[ref.r] + row;
        if (p.accumulate) out += *yp;
        *yp = out;
        if (p.push.world > 0) {
            // the next exchange's epoch (set by the previous exchange, which has
            // ended: read-only while this grid runs, so through the read-only cache)
            const unsigned epoch = __ldg(p.push.ctr) + 1u;
            const size_t off = ((size_t)(epoch & 1u) * p.push.world + p.push.rank) * p.push.slot_elems +
                               (size_t)tok * p.ldys[ref.r] + row;
            for (int r = 0; r < p.push.world; ++r)
                if (r != p.push.rank) st_tagged(p.push.peers.tagged[r] + off, out, epoch);
        }
    } else {
        float gv, uv;
        if (LAYOUT == kLayoutS8) {
            gv = (float)v * (p.src[0].scale * p.sx[tok]);
            uv = (float)v_up * (p.src[1].scale * p.sx[tok]);
        } else {
            gv = ((float)v * kTwo24) * xe[tok];
            uv = ((float)v_up * kTwo24) * xe[tok];
        }
        if (p.src[0].bias) gv += p.src[0].bias[row];
        if (p.src[1].bias) uv += p.src[1].bias[row];
        p.y[(size_t)tok * p.ldy + row] = silu_f(gv) * uv;
    }
}

template <typename Acc> struct Vec4;
template <> struct Vec4<float> {
    using T = float4;
    __device__ static T zero() { return make_float4(0.f, 0.f, 0.f, 0.f); }
    __device__ static void add(T &a, const T &b) { a.x += b.x; a.y += b.y; a.z += b.z; a.w += b.w; }
};
template <> struct Vec4<int> {
    using T = int4;
    __device__ static T zero() { return make_int4(0, 0, 0, 0); }
    __device__ static void add(T &a, const T &b) { a.x += b.x; a.y += b.y; a.z += b.z; a.w += b.w; }
};
template <typename Acc> struct Vec2;
template <> struct Vec2<float> {
    using T = float2;
    __device__ static T zero() { return make_float2(0.f, 0.f); }
    __device__ static void add(T &a, const T &b) { a.x += b.x; a.y += b.y; }
    __device__ static T sum(const T &a, const T &b) { return make_float2(a.x + b.x, a.y + b.y); }
};
template <> struct Vec2<int> {
    using T = int2;
    __device__ static T zero() { return make_int2(0, 0); }
    __device__ static void add(T &a, const T &b) { a.x += b.x; a.y += b.y; }
    __device__ static T sum(const T &a, const T &b) { return make_int2(a.x + b.x, a.y + b.y); }
};

// Final sum of the ctot chunk slots of strip group sg (slots [ctot][nq]
// entries, nq = kSG * 16 * M), finalized into y: eight running sums over the
// chunks (chunk c into sum c % 8), combined as
// ((s0 + s1) + (s2 + s3)) + ((s4 + s5) + (s6 + s7)).  The association depends
// only on ctot, so the result does not depend on which CTA runs it.  Two
// entries per lane and load.
template <int LAYOUT, int MODE, typename Acc>
__device__ __forceinline__ void reduce_slots(const GemvParams &p, const Acc *slots, int ctot, int sg, int lane,
                                             const float *xe) {
    using V2 = Vec2<Acc>;
    using T2 = typename V2::T;
    const int M = p.M;
    const int nq2 = kSG * 16 * M / 2;             // float2 units of a slot
    const int nout2 = MODE == 1 ? nq2 / 2 : nq2;  // units finalized (gate/up: the gate half)
    const int up2 = 16 * M;                       // gate/up: up entries follow two strips later
    const T2 *s2 = reinterpret_cast<const T2 *>(slots);
    for (int q2 = lane; q2 < nout2; q2 += 32) {
        T2 a[8], u[8];
#pragma unroll
        for (int h = 0; h < 8; ++h) a[h] = u[h] = V2::zero();
        int c = 0;
        for (; c + 8 <= ctot; c += 8) {
#pragma unroll
            for (int h = 0; h < 8; ++h) {
                V2::add(a[h], __ldcg(&s2[(size_t)(c + h) * nq2 + q2]));
                if (MODE == 1) V2::add(u[h], __ldcg(&s2[(size_t)(c + h) * nq2 + q2 + up2]));
            }
        }
#pragma unroll
        for (int h = 0; h < 7; ++h)
            if (c + h < ctot) {
                V2::add(a[h], __ldcg(&s2[(size_t)(c + h) * nq2 + q2]));
                if (MODE == 1) V2::add(u[h], __ldcg(&s2[(size_t)(c + h) * nq2 + q2 + up2]));
            }
        const T2 v = V2::sum(V2::sum(V2::sum(a[0], a[1]), V2::sum(a[2], a[3])),
                             V2::sum(V2::sum(a[4], a[5]), V2::sum(a[6], a[7])));
        const T2 vu = V2::sum(V2::sum(V2::sum(u[0], u[1]), V2::sum(u[2], u[3])),
                              V2::sum(V2::sum(u[4], u[5]), V2::sum(u[6], u[7])));
        finalize_entry<LAYOUT, MODE, Acc>(p, sg, 2 * q2, v.x, vu.x, xe);
        finalize_entry<LAYOUT, MODE, Acc>(p, sg, 2 * q2 + 1, v.y, vu.y, xe);
    }
}

template <typename V> __device__ __forceinline__ auto comp(const V &v, int c) {
    return c == 0 ? v.x : c == 1 ? v.y : c == 2 ? v.z : v.w;
}

// Value k of row m of a fused fill's source, specialised by op (the switch of
// xsrc_value resolved at compile time, so the loads of a unit can be issued
// together).
// (RMSNorm, the op of every block's first GEMV, is resolved at compile time;
// the other ops go through xsrc_value.)
template <int OP>
__device__ __forceinline__ float fused_src(const XSrc &s, int m, int k, float inv) {
    if constexpr (OP == kXRmsnorm) {
        return __fmul_rn(__fmul_rn(static_cast<const float *>(s.x)[(size_t)m * s.ldx + k], inv), s.aux[k]);
    } else {
        return xsrc_value(s, m, k, inv);
    }
}

// Fused fill (fp32 activations split into fp16 hi + lo, F16 layout): the 256
// threads of the MMA warps build this CTA's K-slice of activation fragments
// and epilogue-block sums in shared memory, in the layout the bulk-copied
// fragments have (chpe_xfill_f16_kernel, same bits), straight from the source op --
// RMSNorm statistics included, so no fill kernel runs between two GEMVs.
// Ends with a barrier of the MMA warps.
template <int BITS, int E, int OP>
__device__ __forceinline__ void fused_fill_op(const GemvParams &p, uint8_t *xf_s, float *xs_s, float *scratch,
                                              float *xe_s, int b0, int nb, int span) {
    constexpr int S = (256 / BITS) / 16;  // k-steps per chunk
    const int tid = threadIdx.x;           // 0..255 (MMA warps)
    const int M = p.M, K = p.K;
    const XSrc &xs = p.xsrc;
    // Row statistics over the whole row in the fill kernel's order (the
    // 256 MMA threads play the fill CTA's 512): the RMSNorm scale and the
    // row's power-of-two scale 2^e, so the fragments are the fill kernel's bits.
    float inv[kMaxTokens], scl[kMaxTokens];
    const int nunits = (p.n_blocks * span) / 4;
#pragma unroll
    for (int m = 0; m < kMaxTokens; ++m) {
        inv[m] = 1.0f;
        scl[m] = 1.0f;
        if (m >= M) continue;
        float amax;
        block_row_stats(xs, m, K, nunits, tid, kNW * 32, scratch, 1, inv[m], amax);
        const int e = row_scale_exp(amax);
        scl[m] = pow2_of(e);
        if (tid == 0) {
            xe_s[m] = pow2_of(-e);
            if (blockIdx.x == 0) const_cast<float *>(p.xe)[m] = pow2_of(-e);  // for the chunk-sum kernel
        }
    }
    const int units = nb * kChunksPerBlock * S * 4;  // a multiple of 32: whole warps take part below
    const int k_base = b0 * span;
#pragma unroll 2
    for (int u = tid; u < units; u += kNW * 32) {
        const int sr = u >> 2, t = u & 3;
        const int j = sr % S;
        const int sh = BITS == 4 ? 4 * (j & 1) : BITS == 2 ? 2 * (j & 3) : 0;
        const float down = pow2_of(-sh), up = pow2_of(sh);
        const int kb = k_base + 16 * sr + 2 * t;
        const int kk[4] = {kb, kb + 1, kb + 8, kb + 9};
        float part[kMaxTokens];
#pragma unroll
        for (int m = 0; m < kMaxTokens; ++m) {
            part[m] = 0.0f;
            if (m < M) {
                float v[4];
#pragma unroll
                for (int q = 0; q < 4; ++q) v[q] = kk[q] < K ? fused_src<OP>(xs, m, kk[q], inv[m]) : 0.0f;
                __half h[4], l[4];
                const float dn = scl[m] * down;  // 2^(e - sh), as the fill kernel's pre-scale
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const float w = v[q] * dn;
                    h[q] = __float2half_rn(w);
                    l[q] = __float2half_rn(w - __half2float(h[q]));
                    part[m] += (__half2float(h[q]) + __half2float(l[q])) * up;
                }
                *reinterpret_cast<uint4 *>(xf_s + ((size_t)(sr * M + m) * 4 + t) * 16) =
                    make_uint4(pack_h2(h[0], h[1]), pack_h2(h[2], h[3]), pack_h2(l[0], l[1]), pack_h2(l[2], l[3]));
            }
        }
        // E/4 consecutive threads hold one epilogue block
#pragma unroll
        for (int m = 0; m < kMaxTokens; ++m) {
            if (m >= M) break;
            float v = part[m];
            for (int off = E / 8; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
            if ((u % (E / 4)) == 0) xs_s[(size_t)(u / (E / 4)) * 8 + m] = v;
        }
    }
    named_bar_sync(1, kNW * 32);
}

template <int BITS, int E>
__device__ __forceinline__ void fused_fill(const GemvParams &p, uint8_t *xf_s, float *xs_s, float *scratch,
                                           float *xe_s, int b0, int nb, int span) {
    if (p.xsrc.op == kXRmsnorm)
        fused_fill_op<BITS, E, kXRmsnorm>(p, xf_s, xs_s, scratch, xe_s, b0, nb, span);
    else
        fused_fill_op<BITS, E, -1>(p, xf_s, xs_s, scratch, xe_s, b0, nb, span);
}

// XM: how the activation operand is fed (GemvPlan::xmode).
template <int BITS, int LAYOUT, int E, int XM, int MODE, int META>
__global__ void __launch_bounds__(kThreads, 2) chpe_qgemv_kernel(const GemvParams p) {
    using Acc = typename std::conditional<LAYOUT == kLayoutS8, int, float>::type;
    using V4 = Vec4<Acc>;
    using Acc4 = typename V4::T;
    constexpr bool XSPLIT = XM != 0;
    constexpr int KC = 256 / BITS;
    constexpr int S = (LAYOUT == kLayoutS8) ? 1 : KC / 16;
    constexpr int NE = (LAYOUT == kLayoutS8) ? 1 : KC / E;
    constexpr int SPE = (LAYOUT == kLayoutS8) ? 1 : E / 16;
    constexpr int MB = META == kMetaS16 ? 2 : META == kMetaSZ16 ? 4 : 8;
    constexpr int kLast = 1;  // ring tag: last block of a unit (the chunk index in the bits above)

    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int ks = blockIdx.x % p.n_ks;
    const int jk = blockIdx.x / p.n_ks;
    const int Gk = gridDim.x / p.n_ks;
    const int b0 = ks * p.bpk;
    const int b1 = min(b0 + p.bpk, p.n_blocks);
    const int nb = b1 - b0;
    const int C = unit_chunks(nb, p.bc);                      // chunks per chunked strip group in this slice
    const int U = slice_units(p.n_sg, p.n_whole, C);          // units of this slice
    const int NS = p.nstages;                                 // ring stages (2 or 3)
    const int PS = static_units(p.n_whole, Gk, nb, p.pref, NS);  // static units per CTA
    const int M = p.M;
    const int BB = p.block_bytes;
    const bool XS = p.xstream != 0;  // activations stream through the ring with the weights
    const SmemLayout L = smem_layout(LAYOUT, BITS, p.bpk, M, XSPLIT, E, BB, p.xstream, NS);

    uint64_t *full = reinterpret_cast<uint64_t *>(smem + L.bar);
    uint64_t *empty = full + kStages;
    uint64_t *xbar = empty + kStages;
    uint64_t *rfull = xbar + 1;              // [nbuf] MMA warps -> epilogue warp: accumulators written
    uint64_t *rempty = rfull + kMaxRedBufs;  // [nbuf] epilogue warp -> MMA warps: buffer free again
    const int nbuf = L.nbuf;                 // 2 or 4
    const int nbuf_log = nbuf >> 1;          // log2(nbuf)
    int *tag_unit = reinterpret_cast<int *>(smem + L.tags);
    int *tag_blk = tag_unit + kStages;
    int *tag_flags = tag_blk + kStages;
    SegInfo *info = reinterpret_cast<SegInfo *>(smem + L.info);

    if (threadIdx.x == 0) {
#pragma unroll
        for (int s = 0; s < NS; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kNW);
        }
        mbar_init(xbar, 1);
        for (int b = 0; b < nbuf; ++b) {
            mbar_init(&rfull[b], kNW);  // one arrival per MMA warp
            mbar_init(&rempty[b], 1);
        }
        *reinterpret_cast<uint4 *>(smem + kZeroSlot) = make_uint4(0u, 0u, 0u, 0u);
        fence_barrier_init();
        // the next kernel on the stream may be scheduled now: it waits for
        // this grid before it touches anything this grid reads or writes
        grid_dependents_launch();
    }
    __syncthreads();

    if (warp == kProducerWarp) {
        // ---------------- producer warp ----------------
        // The whole warp runs the loop (uniform control flow): lane 0 draws
        // units, arms the stage barriers and writes the ring tags; lane q < kSG
        // sets up strip q of each unit and issues its copies, so the copies of
        // a stage go out as one warp instruction.  A single thread doing all of
        // it falls behind the MMA warps when units are short.
        const uint64_t pol = l2_policy_evict_first();
        unsigned *wctr = p.work_ctr + ks;
        const int n_grabs = grabs_total(U, PS, Gk);
        int it = 0, slot = 0, use = 0;  // ring position: items issued, slot, pass
        bool x_issued = false;
        const uint32_t xblk = (uint32_t)xfrag_bytes_per_block(LAYOUT, BITS, M, XSPLIT);
        const uint32_t xsblk = LAYOUT == kLayoutF16 ? (uint32_t)(kChunksPerBlock * NE * 32) : 0u;
        int armed = 0;  // stages armed so far (their activations follow the upstream wait)
        // Streamed activations of block bi of the slice into ring slot sl (lanes
        // kSG and kSG + 1; only once the upstream grid has finished).
        auto copy_xblock = [&](int sl, int bi) {
            uint8_t *st = smem + L.ring + (size_t)sl * L.stage;
            const size_t b = (size_t)(b0 + bi);
            if (lane == kSG) bulk_g2s(st + L.sx, static_cast<const uint8_t *>(p.xf) + b * xblk, xblk, &full[sl]);
            if (LAYOUT == kLayoutF16 && lane == kSG + 1)
                bulk_g2s(st + L.sxs, reinterpret_cast<const uint8_t *>(p.xs) + b * xsblk, xsblk, &full[sl]);
        };
        // After the upstream grid has finished: the activations (unless the
        // MMA warps build them) and, from then on, the work counter.
        auto issue_x = [&]() {
            grid_dependency_wait();
            x_issued = true;
            if (XS) {
                // the stages armed before the wait still miss their activations
                // (at most NS of them, slots 0 .. it-1 of the first pass)
                __syncwarp();
                for (int q = 0; q < armed && q < NS; ++q) copy_xblock(q, tag_blk[q]);
                return;
            }
            if (p.fused || lane != 0) return;
            const uint32_t xb = (uint32_t)(nb * xfrag_bytes_per_block(LAYOUT, BITS, M, XSPLIT));
            uint32_t tx = xb;
            const uint32_t xsb = (uint32_t)nb * kChunksPerBlock * NE * 32;
            if (LAYOUT == kLayoutF16) tx += xsb;
            mbar_arrive_expect_tx(xbar, tx);
            bulk_g2s(smem + L.xf,
                     static_cast<const uint8_t *>(p.xf) + (size_t)b0 * xfrag_bytes_per_block(LAYOUT, BITS, M, XSPLIT), xb,
                     xbar);
            if (LAYOUT == kLayoutF16)
                bulk_g2s(smem + L.xs, reinterpret_cast<const uint8_t *>(p.xs) + (size_t)b0 * kChunksPerBlock * NE * 32,
                         xsb, xbar);
        };
        int pi = 0;            // static units taken
        bool pending = false;  // a draw is in flight (lane 0 holds its value)
        unsigned drawn = 0;
        auto draw = [&]() {
            if (pending) return;
            if (!x_issued) issue_x();
            if (lane == 0) drawn = atomicAdd(wctr, 1u);
            pending = true;
        };
        auto static_left = [&]() { return pi < PS && jk + pi * Gk < U; };
        auto next_unit = [&]() -> int {
            if (static_left()) return jk + (pi++) * Gk;
            pi = PS;
            draw();
            pending = false;
            const int d = (int)__shfl_sync(0xffffffffu, drawn, 0);
            const int u = PS * Gk + d;
            if (u < U) return u;
            if (lane == 0 && d == n_grabs - 1) atomicExch(wctr, 0u);  // the launch's last draw
            return -1;
        };
        bool stop = false;
        while (!stop) {
            const int u = next_unit();
            if (u < 0) break;
            const Unit un = unit_of(u, nb, C, ks, p.n_ks, p.n_whole, p.bc, p.cfull, p.ctot);
            const uint8_t *src = nullptr;  // lane q < kSG: strip q, block bs of the unit
            bool valid = false;
            if (lane < kSG) {
                const StripRef r = strip_ref<MODE>(p, un.sg, lane);
                valid = r.valid;
                if (valid) src = p.src[r.r].codes + ((size_t)r.strip * p.n_blocks + b0 + un.bs) * BB;
            }
            const uint32_t tx = (uint32_t)__popc(__ballot_sync(0xffffffffu, valid)) * (uint32_t)BB +
                                (XS ? xblk + xsblk : 0u);
            uint8_t *dst = smem + L.ring + (size_t)lane * BB;
            for (int bi = un.bs; bi < un.be; ++bi, ++it) {
                // the next unit's draw goes out with the first copy of this one,
                // so its L2 round trip overlaps the whole unit
                if (bi == un.bs && !static_left()) draw();
                if (use > 0 && !__all_sync(0xffffffffu, mbar_wait_bounded(&empty[slot], (use - 1) & 1))) {
                    if (lane == 0) atomicExch(p.err, kErrWaitEmpty);
                    stop = true;
                    break;
                }
                if (lane == 0) {
                    tag_unit[slot] = un.sg;
                    tag_blk[slot] = bi;
                    tag_flags[slot] = (bi == un.be - 1 ? kLast : 0) | (un.gc << 1);
                    mbar_arrive_expect_tx(&full[slot], tx);
                }
                __syncwarp();
                if (valid)
                    bulk_g2s_hint(dst + (size_t)slot * L.stage, src + (size_t)(bi - un.bs) * BB, (uint32_t)BB,
                                  &full[slot], pol);
                if (XS && x_issued) copy_xblock(slot, bi);
                ++armed;
                if (++slot == NS) {
                    slot = 0;
                    ++use;
                }
                // weights first, then (once) the upstream-dependent activations
                if (!x_issued && it + 1 >= NS) issue_x();
            }
        }
        if (!x_issued) issue_x();
        if (lane == 0) {
            // end-of-work marker in the next slot
            if (use > 0 && !mbar_wait_bounded(&empty[slot], (use - 1) & 1)) atomicExch(p.err, kErrWaitEmpty);
            tag_unit[slot] = -1;
            mbar_arrive(&full[slot]);
            ++it;
            // every issued copy has landed before the CTA may exit
            for (int s = 0; s < NS && s < it; ++s) {
                const int last = s + ((it - 1 - s) / NS) * NS;
                if (!mbar_wait_bounded(&full[s], (last / NS) & 1)) atomicExch(p.err, kErrWaitFull);
            }
            if (!p.fused && !XS && !mbar_wait_bounded(xbar, 0)) atomicExch(p.err, kErrWaitPrologue);
        }
    } else if (warp == kEpilogueWarp) {
        // ---------------- epilogue warp ----------------
        // Sums the MMA warps' accumulators of each finished unit (fixed warp
        // order, four entries per load).  A strip group whose K is one unit is
        // written out here; otherwise the sum goes to the unit's chunk slot and
        // the arrival count of the strip group is raised (acquire-release); the
        // arrival that completes the count sums all chunk slots and writes the
        // outputs (with rmode 1 chpe_qgemv_reduce_kernel does, after this kernel).
        // Runs behind the MMA warps, off the streaming path.
        grid_dependency_wait();  // y, the workspace and the counters belong to the previous grid until it ends
        Acc *ws = static_cast<Acc *>(p.ws);
        // row unscale factors: the fill's (global), or this CTA's fused fill's
        // (shared; written before the first unit is handed over)
        const float *xe = p.fused ? reinterpret_cast<const float *>(smem + L.xe) : p.xe;
        const int nq = kSG * 16 * M;  // (strip, row, token) entries of a unit
        const int nq4 = nq / 4;       // nq is a multiple of 64
        for (int k = 0;; ++k) {
            const int b = k & (nbuf - 1), u = k >> nbuf_log;
            if (!__all_sync(0xffffffffu, mbar_wait_bounded(&rfull[b], u & 1))) {
                if (lane == 0) atomicExch(p.err, kErrWaitFull);
                break;
            }
            const SegInfo si = info[b];
            if (si.sg < 0) break;
            const int sg = si.sg;
            const Acc4 *red4 = reinterpret_cast<const Acc4 *>(smem + L.red) + (size_t)b * kNW * nq4;
            const int ctot = sg < p.n_whole ? p.n_ks : p.ctot;  // chunks of this strip group
            if (ctot == 1) {
                // gate/up: entry q of a gate strip pairs with q + 2*16*M of the up strip
                const int nq4_out = MODE == 1 ? nq4 / 2 : nq4;
                const int up4 = 2 * 16 * M / 4;
                for (int q4 = lane; q4 < nq4_out; q4 += 32) {
                    Acc4 sum = V4::zero(), su = V4::zero();
#pragma unroll
                    for (int w = 0; w < kNW; ++w) {
                        V4::add(sum, red4[(size_t)w * nq4 + q4]);
                        if (MODE == 1) V4::add(su, red4[(size_t)w * nq4 + q4 + up4]);
                    }
#pragma unroll
                    for (int c = 0; c < 4; ++c)
                        finalize_entry<LAYOUT, MODE, Acc>(p, sg, 4 * q4 + c, comp(sum, c), comp(su, c), xe);
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&rempty[b]);  // accumulator buffer consumed
                continue;
            }
            Acc *slots = ws + (size_t)sg * p.ctot * nq;
            Acc4 *wslot4 = reinterpret_cast<Acc4 *>(slots + (size_t)si.gc * nq);
            for (int q4 = lane; q4 < nq4; q4 += 32) {
                Acc4 sum = V4::zero();
#pragma unroll
                for (int w = 0; w < kNW; ++w) V4::add(sum, red4[(size_t)w * nq4 + q4]);
                wslot4[q4] = sum;
            }
            __syncwarp();
            if (p.rmode == 1) {  // chpe_qgemv_reduce_kernel sums the slots after this kernel
                if (lane == 0) mbar_arrive(&rempty[b]);
                continue;
            }
            unsigned old = 0;
            if (lane == 0) {
                mbar_arrive(&rempty[b]);  // accumulator buffer consumed
                old = atom_add_acq_rel_gpu(&p.split_cnt[sg], 1u);
            }
            old = __shfl_sync(0xffffffffu, old, 0);
            if (old != (unsigned)(ctot - 1)) continue;
            __syncwarp();
            // the last chunk of strip group sg to arrive: every slot is written
            reduce_slots<LAYOUT, MODE, Acc>(p, slots, ctot, sg, lane, xe);
            __syncwarp();
            if (lane == 0) p.split_cnt[sg] = 0u;  // clean for the next launch
        }
    } else {
        // ---------------- MMA warps ----------------
        const int g = lane >> 2, t = lane & 3;
        // Lane (g, t) supplies column g of the MMA's B operand: token g (XM 0, 1,
        // S8 layout), or token g / 2, fp16 half g & 1 of the fp32 activation
        // (XM 2; the two halves of one token meet again in d[0] + d[1]).  Lanes
        // past the last column read 16 zero bytes (stride 0) instead.
        constexpr bool PK = XM == 2;
        const bool has_x = g < (PK ? 2 * M : M);
        uint32_t xlane;  // this lane's byte offset inside a fragment unit
        uint32_t xstr;   // bytes per fragment unit (k-step, k-step pair, or S8 chunk)
        if (LAYOUT == kLayoutS8) {
            xlane = (g * 4 + t) * 8;
            xstr = (uint32_t)M * 32;
        } else if (PK) {
            xlane = ((g >> 1) * 4 + t) * 16 + (g & 1) * 8;
            xstr = (uint32_t)M * 64;
        } else {
            xlane = (g * 4 + t) * 16;
            xstr = (uint32_t)M * 64;
        }
        if (!has_x) xstr = 0;
        // resident activations: the slice's fragments; streamed: the stage's block
        const uint8_t *xres = has_x ? smem + L.xf + xlane : smem + kZeroSlot;
        const float *xss_res = reinterpret_cast<const float *>(smem + L.xs);
        float zc24[kSG];
#pragma unroll
        for (int i = 0; i < kSG; ++i) zc24[i] = -p.src[source_of<MODE>(i)].zc * kTwoM24;
        const int gshift = p.gshift;

        bool aborted = false;
        if constexpr (LAYOUT == kLayoutF16 && XSPLIT) {
            if (p.fused) {
                grid_dependency_wait();  // the source rows are the previous kernel's output
                fused_fill<BITS, E>(p, smem + L.xf, reinterpret_cast<float *>(smem + L.xs),
                                    reinterpret_cast<float *>(smem + L.red), reinterpret_cast<float *>(smem + L.xe),
                                    b0, nb, KC * kChunksPerBlock);
            }
        }
        if (!p.fused && !XS) {
            // A timed-out wait ends this warp's work; decisions are taken per warp
            // (__all_sync) and every wait is bounded, so no warp can be left stuck.
            if (!__all_sync(0xffffffffu, mbar_wait_bounded(xbar, 0))) {
                if (lane == 0) atomicExch(p.err, kErrWaitPrologue);
                aborted = true;
            }
            grid_dependency_wait();
        }

        Acc acc[kSG][4];
#pragma unroll
        for (int i = 0; i < kSG; ++i)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[i][e] = 0;
        int nseg = 0;
        // Hands the accumulators (or the end-of-work mark, sg < 0) to the epilogue warp.
        auto hand_off = [&](int sg, int gc) -> bool {
            const int b = nseg & (nbuf - 1), u = nseg >> nbuf_log;
            if (u > 0 && !__all_sync(0xffffffffu, mbar_wait_bounded(&rempty[b], (u - 1) & 1))) {
                if (lane == 0) atomicExch(p.err, kErrWaitEmpty);
                return false;
            }
            Acc *red = reinterpret_cast<Acc *>(smem + L.red) + ((size_t)b * kNW + warp) * kSG * 16 * M;
            // XM 2: lane (g, t) holds rows g (e = 0) and g + 8 (e = 1) of token t;
            // otherwise rows g (e = 0, 1) and g + 8 (e = 2, 3), tokens 2t + (e & 1)
#pragma unroll
            for (int i = 0; i < kSG; ++i)
#pragma unroll
                for (int e = 0; e < (PK ? 2 : 4); ++e) {
                    const int tok = PK ? t : 2 * t + (e & 1);
                    const int r = PK ? g + 8 * e : g + 8 * (e >> 1);
                    if (tok < M) red[(i * 16 + r) * M + tok] = acc[i][e];
                    acc[i][e] = 0;
                }
            if (warp == 0 && lane == 0) info[b] = SegInfo{sg, gc};
            // one arrival per warp, after its stores
            __syncwarp();
            if (lane == 0) mbar_arrive(&rfull[b]);
            ++nseg;
            return true;
        };

        int slot = 0, use = 0;
        for (;; ) {
            if (aborted) break;
            if (!__all_sync(0xffffffffu, mbar_wait_bounded(&full[slot], use & 1))) {
                if (lane == 0) atomicExch(p.err, kErrWaitFull);
                aborted = true;
                break;
            }
            const int sg = tag_unit[slot];
            if (sg < 0) break;
            const int bi = tag_blk[slot];
            const int flags = tag_flags[slot];
            const uint8_t *stg = smem + L.ring + (size_t)slot * L.stage;
            // chunk of the activations' array: in the slice (resident) or in the stage's block (streamed)
            const int cs = XS ? warp : bi * kChunksPerBlock + warp;
            const uint8_t *xb0 = XS ? (has_x ? stg + L.sx + xlane : smem + kZeroSlot) : xres;
            const float *xss = XS ? reinterpret_cast<const float *>(stg + L.sxs) : xss_res;
            uint4 wv[kSG];
#pragma unroll
            for (int i = 0; i < kSG; ++i)
                wv[i] = *reinterpret_cast<const uint4 *>(stg + (size_t)i * BB + warp * kChunkBytes + lane * 16);
            if constexpr (LAYOUT == kLayoutS8) {
                const uint2 b = *reinterpret_cast<const uint2 *>(xb0 + (uint32_t)cs * xstr);
#pragma unroll
                for (int i = 0; i < kSG; ++i)
                    mma_s8_m16n8k32(reinterpret_cast<int *>(acc[i]), wv[i].x, wv[i].y, wv[i].z, wv[i].w, b.x, b.y);
            } else {
                uint4 w8[kSG];
#pragma unroll
                for (int i = 0; i < kSG; ++i)
                    w8[i] = (BITS == 8) ? wv[i]
                                        : make_uint4(wv[i].x >> 8, wv[i].y >> 8, wv[i].z >> 8, wv[i].w >> 8);
#pragma unroll
                for (int eb = 0; eb < NE; ++eb) {
                    float d[kSG][4];
#pragma unroll
                    for (int i = 0; i < kSG; ++i)
#pragma unroll
                        for (int e = 0; e < 4; ++e) d[i][e] = 0.0f;
#pragma unroll
                    for (int jj = 0; jj < SPE; jj += (XM == 0 ? 2 : 1)) {
                        const int j = eb * SPE + jj;
                        const int kst = cs * S + j;
                        if constexpr (XM == 2) {
                            const uint2 bv = *reinterpret_cast<const uint2 *>(xb0 + (uint32_t)kst * xstr);
#pragma unroll
                            for (int i = 0; i < kSG; ++i)
                                mma_f16_m16n8k16(d[i], unpack_f16<BITS>(wv[i].x, w8[i].x, j),
                                                 unpack_f16<BITS>(wv[i].y, w8[i].y, j),
                                                 unpack_f16<BITS>(wv[i].z, w8[i].z, j),
                                                 unpack_f16<BITS>(wv[i].w, w8[i].w, j), bv.x, bv.y);
                        } else {
                            const uint4 bv =
                                *reinterpret_cast<const uint4 *>(xb0 + (uint32_t)(XM == 1 ? kst : (kst >> 1)) * xstr);
#pragma unroll
                            for (int i = 0; i < kSG; ++i) {
                                mma_f16_m16n8k16(d[i], unpack_f16<BITS>(wv[i].x, w8[i].x, j),
                                                 unpack_f16<BITS>(wv[i].y, w8[i].y, j),
                                                 unpack_f16<BITS>(wv[i].z, w8[i].z, j),
                                                 unpack_f16<BITS>(wv[i].w, w8[i].w, j), bv.x, bv.y);
                                const int j2 = XM == 1 ? j : j + 1;
                                mma_f16_m16n8k16(d[i], unpack_f16<BITS>(wv[i].x, w8[i].x, j2),
                                                 unpack_f16<BITS>(wv[i].y, w8[i].y, j2),
                                                 unpack_f16<BITS>(wv[i].z, w8[i].z, j2),
                                                 unpack_f16<BITS>(wv[i].w, w8[i].w, j2), bv.z, bv.w);
                            }
                        }
                    }
                    const int kib = warp * KC + eb * E;  // column within the block
                    const int gib = gshift >= 0 ? (kib >> gshift) : 0;
                    if constexpr (XM == 2) {
                        const float X = xss[((size_t)cs * NE + eb) * 8 + t];
#pragma unroll
                        for (int i = 0; i < kSG; ++i) {
                            float s0, o0, s1, o1;
                            load_meta2<META>(stg + (size_t)i * BB + kBlockCodeBytes + (size_t)gib * 16 * MB, g,
                                             zc24[i], s0, o0, s1, o1);
                            acc[i][0] = fmaf(o0, X, fmaf(s0, d[i][0] + d[i][1], acc[i][0]));
                            acc[i][1] = fmaf(o1, X, fmaf(s1, d[i][2] + d[i][3], acc[i][1]));
                        }
                    } else {
                        const float2 X = *reinterpret_cast<const float2 *>(xss + ((size_t)cs * NE + eb) * 8 + 2 * t);
#pragma unroll
                        for (int i = 0; i < kSG; ++i) {
                            float s0, o0, s1, o1;
                            load_meta2<META>(stg + (size_t)i * BB + kBlockCodeBytes + (size_t)gib * 16 * MB, g,
                                             zc24[i], s0, o0, s1, o1);
                            acc[i][0] = fmaf(o0, X.x, fmaf(s0, d[i][0], acc[i][0]));
                            acc[i][1] = fmaf(o0, X.y, fmaf(s0, d[i][1], acc[i][1]));
                            acc[i][2] = fmaf(o1, X.x, fmaf(s1, d[i][2], acc[i][2]));
                            acc[i][3] = fmaf(o1, X.y, fmaf(s1, d[i][3], acc[i][3]));
                        }
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
            if (++slot == NS) {
                slot = 0;
                ++use;
            }
            if (flags & kLast) {
                if (!hand_off(sg, flags >> 1)) {
                    aborted = true;
                    break;
                }
            }
        }
        if (!aborted) hand_off(-1, 0);  // end of work for the epilogue warp
    }
    __syncthreads();
}

// rmode 1: sums the chunk slots of every chunked strip group in chunk order
// (reduce_slots: the association of the in-kernel path) and writes its
// outputs; one warp per strip group.  With more than two rows an arrival
// count per unit would keep the epilogue warp waiting on L2 round trips,
// and through it the MMA warps.
template <int LAYOUT, int MODE>
__global__ void __launch_bounds__(128) chpe_qgemv_reduce_kernel(const GemvParams p) {
    using Acc = typename std::conditional<LAYOUT == kLayoutS8, int, float>::type;
    pdl_begin();
    const int lane = threadIdx.x & 31;
    const int nq = kSG * 16 * p.M;
    for (int sg = blockIdx.x * 4 + (threadIdx.x >> 5); sg < p.n_sg; sg += gridDim.x * 4) {
        const int ctot = sg < p.n_whole ? p.n_ks : p.ctot;
        if (ctot == 1) continue;  // finished by the GEMV kernel
        reduce_slots<LAYOUT, MODE, Acc>(p, static_cast<const Acc *>(p.ws) + (size_t)sg * p.ctot * nq, ctot, sg,
                                        lane, p.xe);
    }
}

template <int BITS, int LAYOUT, int E, int XM, int MODE, int META>
cudaError_t launch_gemv_t(const GemvPlan &plan, const GemvParams &p_in, cudaStream_t st) {
    auto kern = chpe_qgemv_kernel<BITS, LAYOUT, E, XM, MODE, META>;
    // one wave of resident CTAs: the planned grid capped by the real occupancy
    // (queried once per device and shared-memory size; the registers are fixed)
    static KernelDeviceState kstate;
    int occ = 1;
    cudaError_t pe = kernel_prepare(kstate, kern, kThreads, kSmemBudget, plan.smem, &occ);
    if (pe != cudaSuccess) return pe;
    long gk = std::min<long>((long)plan.sms * occ / plan.n_ks, plan.items_min);
    gk = std::max<long>(1, std::min<long>(gk, plan.grid / plan.n_ks));
    GemvParams p = p_in;
    p.gk = (int)gk;
    p.rmode = plan.rmode;
    p.xstream = plan.xstream;
    p.nstages = plan.nstages;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(gk * plan.n_ks));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = plan.smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    note_launch();
    cudaError_t e = cudaLaunchKernelEx(&cfg, kern, p);
    if (e != cudaSuccess || !plan.rmode || plan.ctot == 1) return e;
    // the chunk sums, on the same stream right behind
    cudaLaunchConfig_t rc = cfg;
    rc.gridDim = dim3((unsigned)std::min<long>((p.n_sg + 3) / 4, (long)plan.sms * 4));
    rc.blockDim = dim3(128);
    rc.dynamicSmemBytes = 0;
    note_launch();
    return cudaLaunchKernelEx(&rc, chpe_qgemv_reduce_kernel<LAYOUT, MODE>, p);
}

// All variants of one code width / epilogue block, chosen at run time.
template <int BITS, int LAYOUT, int E>
cudaError_t launch_gemv_bits(const GemvPlan &plan, const GemvParams &p, int meta, cudaStream_t st) {
    if constexpr (LAYOUT == kLayoutS8) {
        if (plan.mode == 0) return launch_gemv_t<BITS, LAYOUT, E, 0, 0, kMetaNone>(plan, p, st);
        return launch_gemv_t<BITS, LAYOUT, E, 0, 1, kMetaNone>(plan, p, st);
    } else {
#define CHPE_META_CASES(XM, MD)                                                                 \
    switch (meta) {                                                                             \
    case kMetaS16: return launch_gemv_t<BITS, LAYOUT, E, XM, MD, kMetaS16>(plan, p, st);        \
    case kMetaSZ16: return launch_gemv_t<BITS, LAYOUT, E, XM, MD, kMetaSZ16>(plan, p, st);      \
    default: return launch_gemv_t<BITS, LAYOUT, E, XM, MD, kMetaF32>(plan, p, st);              \
    }
#define CHPE_XM_CASES(MD)                                                                       \
    switch (plan.xmode) {                                                                       \
    case 2: CHPE_META_CASES(2, MD)                                                              \
    case 1: CHPE_META_CASES(1, MD)                                                              \
    default: CHPE_META_CASES(0, MD)                                                             \
    }
        if (plan.mode == 0) {
            CHPE_XM_CASES(0)
        } else {
            CHPE_XM_CASES(1)
        }
#undef CHPE_XM_CASES
#undef CHPE_META_CASES
    }
}

}  // namespace chpe
