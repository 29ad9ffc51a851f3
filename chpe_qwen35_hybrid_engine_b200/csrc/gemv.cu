// gemv.cu -- decode/verify GEMV for M = 1..8 activation rows over quantized
// weights in the strip layout (layout.h).
//
// One CTA = 4 consumer warps + 1 producer warp and owns a unit of work: two
// 16-row strips (or, for the fused gate/up SwiGLU, the same strip of the gate
// and of the up matrix) over one K-slice.  The producer thread streams the
// unit's 512-byte chunks into a 6-stage shared-memory ring with 1-D bulk
// copies (TMA engine, mbarrier completion, L2 evict-first), after first
// issuing the weight stages and only then waiting on the upstream grid
// (programmatic dependent launch) for the activation fragments.  Consumer
// warps take one chunk per stage, turn codes into fp16 operands in registers
// with one LOP3 / PRMT per pair (the code as an exact fp16 subnormal), issue
// m16n8k16 MMAs against the staged activation fragments, and fold the
// per-group scale / zero-point into fp32 register accumulators:
//     acc += (s * 2^24) * D + (-z * s) * sum(x over the block).
// The int8 x int8 path (W8A8) feeds raw codes to m16n8k32 integer MMAs and
// keeps exact int32 sums.  Warps reduce through shared memory in a fixed
// order; split-K partials go to a workspace and the last CTA of a strip group
// (atomic ticket) sums them in slice order, so results are deterministic.
#include <algorithm>
#include <type_traits>

#include "common.cuh"
#include "internal.h"

namespace chpe {

constexpr int kNW = 4;      // consumer warps per CTA
constexpr int kStages = 6;  // ring depth
constexpr int kSG = 2;      // strips per unit
constexpr int kThreads = (kNW + 1) * 32;
constexpr int kXMaxBytes = 64 * 1024;  // activation fragments staged per CTA
constexpr int kTargetUnits = 4 * 148;

struct SmemLayout {
    size_t bar, ring, xf, xlo, xs, meta, red, flag, total;
};

__host__ __device__ inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

__host__ __device__ inline SmemLayout smem_layout(int layout, int bits, int cpk, int M, bool xsplit, int e_cols,
                                                  int gps, int meta_kind) {
    SmemLayout L;
    size_t o = 0;
    L.bar = 0;
    o = 128;
    L.ring = o;
    o += (size_t)kStages * kSG * kNW * kChunkBytes;
    const int kc = 256 / bits;
    const int steps = layout == kLayoutS8 ? 1 : kc / 16;
    const size_t xb = (size_t)cpk * steps * M * 32;
    L.xf = o;
    o = align_up(o + xb, 128);
    L.xlo = o;
    if (xsplit) o = align_up(o + xb, 128);
    L.xs = o;
    if (layout == kLayoutF16) o = align_up(o + (size_t)cpk * (kc / e_cols) * 32, 128);
    L.meta = o;
    o = align_up(o + (size_t)kSG * gps * 16 * meta_bytes(meta_kind), 128);
    L.red = o;
    o += (size_t)kNW * kSG * 32 * 4 * 4;
    L.flag = o;
    o += 16;
    L.total = align_up(o, 128);
    return L;
}

// Codes become fp16 operands with the exponent field left at zero: the bit
// pattern `code` is the fp16 subnormal code * 2^-24, exact for every code
// (code < 1024).  One LOP3 (4/2-bit) or PRMT (8-bit) yields two operands and
// no subtraction is needed; the 2^24 is folded into the group scale.  The
// accumulator then carries sum(code * x) only, so a small result next to a
// large zero-point term keeps fp32 precision.
template <int BITS>
__device__ __forceinline__ uint32_t unpack_f16(uint32_t w, int j) {
    if constexpr (BITS == 4) {
        return (w >> (4 * j)) & 0x000F000Fu;
    } else if constexpr (BITS == 2) {
        return (w >> (2 * j)) & 0x00030003u;
    } else {
        return __byte_perm(w, 0u, j == 0 ? 0x4140 : 0x4342);
    }
}

constexpr float kTwo24 = 16777216.0f;

// (scale * 2^24, offset per unit of x) of one row-group.
__device__ __forceinline__ void load_meta(int kind, const uint8_t *base, int row, float zc, float &s, float &o) {
    if (kind == kMetaS16) {
        const float sc = __half2float(reinterpret_cast<const __half *>(base)[row]);
        s = sc * kTwo24;
        o = -sc * zc;
    } else if (kind == kMetaSZ16) {
        const __half2 h = reinterpret_cast<const __half2 *>(base)[row];
        const float sc = __low2float(h);
        s = sc * kTwo24;
        o = -sc * __high2float(h);
    } else {
        const float2 f = reinterpret_cast<const float2 *>(base)[row];
        s = f.x * kTwo24;
        o = f.y;
    }
}

template <int BITS, int LAYOUT, int E, bool XSPLIT, int MODE>
__global__ void __launch_bounds__(kThreads) gemv_kernel(const GemvParams p) {
    using Acc = typename std::conditional<LAYOUT == kLayoutS8, int, float>::type;
    constexpr int KC = 256 / BITS;
    constexpr int S = (LAYOUT == kLayoutS8) ? 1 : KC / 16;
    constexpr int NE = (LAYOUT == kLayoutS8) ? 1 : KC / E;
    constexpr int SPE = (LAYOUT == kLayoutS8) ? 1 : E / 16;
    constexpr int MB = 8;  // max metadata entry bytes (float2)

    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int unit = blockIdx.x;
    const int sg = unit / p.n_ks, ks = unit - (unit / p.n_ks) * p.n_ks;
    const int c0 = ks * p.cpk;
    const int c1 = min(c0 + p.cpk, p.n_chunks);
    const int n_c = c1 - c0;
    const int M = p.M;
    const int n_stages = (n_c + kNW - 1) / kNW;

    int strip[kSG];
    bool valid[kSG];
#pragma unroll
    for (int i = 0; i < kSG; ++i) {
        strip[i] = MODE == 1 ? sg : sg * kSG + i;
        valid[i] = strip[i] < p.n_strips;
    }

    int g0 = 0, ng_s = 1;
    if (LAYOUT == kLayoutF16 && p.n_groups > 1) {
        g0 = (c0 * KC) >> p.group_shift;
        const int g1 = min(p.n_groups, ((c1 * KC - 1) >> p.group_shift) + 1);
        ng_s = g1 - g0;
    }
    const int mbytes = meta_bytes(p.meta_kind);
    const SmemLayout L = smem_layout(LAYOUT, BITS, p.cpk, M, XSPLIT, E, p.gps, p.meta_kind);

    uint64_t *full = reinterpret_cast<uint64_t *>(smem + L.bar);
    uint64_t *empty = full + kStages;
    uint64_t *pro = empty + kStages;
    int *s_flag = reinterpret_cast<int *>(smem + L.flag);

    if (threadIdx.x == 0) {
#pragma unroll
        for (int s = 0; s < kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kNW);
        }
        mbar_init(pro, 1);
        fence_barrier_init();
    }
    __syncthreads();

    if (warp == kNW) {
        // ---------------- producer ----------------
        if (lane == 0) {
            const uint64_t pol = l2_policy_evict_first();
            bool ok = true;
            int it = 0;
            auto issue_stage = [&](int i_st) -> bool {
                const int slot = i_st % kStages, use = i_st / kStages;
                if (use > 0 && !mbar_wait_bounded(&empty[slot], (use - 1) & 1)) {
                    atomicExch(p.err, kErrWaitEmpty);
                    return false;
                }
                const int nc = min(kNW, n_c - i_st * kNW);
                uint32_t tx = 0;
#pragma unroll
                for (int i = 0; i < kSG; ++i)
                    if (valid[i]) tx += (uint32_t)nc * kChunkBytes;
                mbar_arrive_expect_tx(&full[slot], tx);
#pragma unroll
                for (int i = 0; i < kSG; ++i) {
                    if (!valid[i]) continue;
                    const uint8_t *src = p.src[MODE == 1 ? i : 0].codes +
                                         ((size_t)strip[i] * p.n_chunks + c0 + (size_t)i_st * kNW) * kChunkBytes;
                    bulk_g2s_hint(smem + L.ring + ((size_t)slot * kSG + i) * kNW * kChunkBytes, src,
                                  (uint32_t)nc * kChunkBytes, &full[slot], pol);
                }
                return true;
            };
            // Weights do not depend on the upstream kernel: start them first.
            for (; it < n_stages && it < kStages && ok; ++it) ok = issue_stage(it);
            grid_dependency_wait();
            {
                uint32_t tx = 0;
                const uint32_t xb = (uint32_t)n_c * S * M * 32;
                tx += xb;
                if (XSPLIT) tx += xb;
                if (LAYOUT == kLayoutF16) tx += (uint32_t)n_c * NE * 32;
                uint32_t mb = (uint32_t)ng_s * 16 * mbytes;
                if (LAYOUT == kLayoutF16)
#pragma unroll
                    for (int i = 0; i < kSG; ++i)
                        if (valid[i]) tx += mb;
                mbar_arrive_expect_tx(pro, tx);
                const size_t xoff = (size_t)c0 * S * M * 32;
                bulk_g2s(smem + L.xf, static_cast<const uint8_t *>(p.xf) + xoff, xb, pro);
                if (XSPLIT) bulk_g2s(smem + L.xlo, static_cast<const uint8_t *>(p.xlo) + xoff, xb, pro);
                if (LAYOUT == kLayoutF16) {
                    bulk_g2s(smem + L.xs, reinterpret_cast<const uint8_t *>(p.xs) + (size_t)c0 * NE * 32,
                             (uint32_t)n_c * NE * 32, pro);
#pragma unroll
                    for (int i = 0; i < kSG; ++i) {
                        if (!valid[i]) continue;
                        const uint8_t *msrc = static_cast<const uint8_t *>(p.src[MODE == 1 ? i : 0].meta) +
                                              ((size_t)strip[i] * p.n_groups + g0) * 16 * mbytes;
                        bulk_g2s(smem + L.meta + (size_t)i * p.gps * 16 * mbytes, msrc, mb, pro);
                    }
                }
            }
            for (; it < n_stages && ok; ++it) ok = issue_stage(it);
            // Drain: every issued stage has landed before the CTA may exit.
            for (int s = 0; s < kStages && s < it; ++s) {
                const int last = s + ((it - 1 - s) / kStages) * kStages;
                if (!mbar_wait_bounded(&full[s], (last / kStages) & 1)) atomicExch(p.err, kErrWaitFull);
            }
            if (!mbar_wait_bounded(pro, 0)) atomicExch(p.err, kErrWaitPrologue);
        }
        return;
    }

    // ---------------- consumers ----------------
    const int g = lane >> 2, t = lane & 3;
    bool aborted = false;
    if (!mbar_wait_bounded(pro, 0)) {
        if (lane == 0) atomicExch(p.err, kErrWaitPrologue);
        aborted = true;
    }
    Acc acc[kSG][4];
#pragma unroll
    for (int i = 0; i < kSG; ++i)
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[i][e] = 0;

    const uint2 *xfs = reinterpret_cast<const uint2 *>(smem + L.xf);
    const uint2 *xls = reinterpret_cast<const uint2 *>(smem + L.xlo);
    const float *xss = reinterpret_cast<const float *>(smem + L.xs);
    float zc[kSG];
#pragma unroll
    for (int i = 0; i < kSG; ++i) zc[i] = p.src[MODE == 1 ? i : 0].zc;

    for (int it = 0; it < n_stages && !aborted; ++it) {
        const int slot = it % kStages, use = it / kStages;
        if (!mbar_wait_bounded(&full[slot], use & 1)) {
            if (lane == 0) atomicExch(p.err, kErrWaitFull);
            aborted = true;
            break;
        }
        const int c = it * kNW + warp;
        if (c < n_c) {
            const uint8_t *stg = smem + L.ring + (size_t)slot * kSG * kNW * kChunkBytes;
            uint4 wv[kSG];
#pragma unroll
            for (int i = 0; i < kSG; ++i)
                wv[i] = *reinterpret_cast<const uint4 *>(stg + ((size_t)i * kNW + warp) * kChunkBytes + lane * 16);
            if constexpr (LAYOUT == kLayoutS8) {
                uint2 b = make_uint2(0u, 0u);
                if (g < M) b = xfs[((size_t)c * M + g) * 4 + t];
#pragma unroll
                for (int i = 0; i < kSG; ++i)
                    mma_s8_m16n8k32(reinterpret_cast<int *>(acc[i]), wv[i].x, wv[i].y, wv[i].z, wv[i].w, b.x, b.y);
            } else {
#pragma unroll
                for (int eb = 0; eb < NE; ++eb) {
                    float d[kSG][4];
#pragma unroll
                    for (int i = 0; i < kSG; ++i)
#pragma unroll
                        for (int e = 0; e < 4; ++e) d[i][e] = 0.0f;
#pragma unroll
                    for (int jj = 0; jj < SPE; ++jj) {
                        const int j = eb * SPE + jj;
                        const size_t kst = (size_t)c * S + j;
                        uint2 b = make_uint2(0u, 0u), bl = make_uint2(0u, 0u);
                        if (g < M) {
                            b = xfs[(kst * M + g) * 4 + t];
                            if (XSPLIT) bl = xls[(kst * M + g) * 4 + t];
                        }
#pragma unroll
                        for (int i = 0; i < kSG; ++i) {
                            const uint32_t a0 = unpack_f16<BITS>(wv[i].x, j);
                            const uint32_t a1 = unpack_f16<BITS>(wv[i].y, j);
                            const uint32_t a2 = unpack_f16<BITS>(wv[i].z, j);
                            const uint32_t a3 = unpack_f16<BITS>(wv[i].w, j);
                            mma_f16_m16n8k16(d[i], a0, a1, a2, a3, b.x, b.y);
                            if (XSPLIT) mma_f16_m16n8k16(d[i], a0, a1, a2, a3, bl.x, bl.y);
                        }
                    }
                    const int kabs = (c0 + c) * KC + eb * E;
                    int gi = (p.n_groups == 1) ? 0 : min(kabs >> p.group_shift, p.n_groups - 1);
                    gi -= g0;
                    const float X0 = xss[((size_t)c * NE + eb) * 8 + 2 * t];
                    const float X1 = xss[((size_t)c * NE + eb) * 8 + 2 * t + 1];
#pragma unroll
                    for (int i = 0; i < kSG; ++i) {
                        const uint8_t *mbase = smem + L.meta + ((size_t)i * p.gps + gi) * 16 * mbytes;
                        float s0, o0, s1, o1;
                        load_meta(p.meta_kind, mbase, g, zc[i], s0, o0);
                        load_meta(p.meta_kind, mbase, g + 8, zc[i], s1, o1);
                        acc[i][0] = fmaf(o0, X0, fmaf(s0, d[i][0], acc[i][0]));
                        acc[i][1] = fmaf(o0, X1, fmaf(s0, d[i][1], acc[i][1]));
                        acc[i][2] = fmaf(o1, X0, fmaf(s1, d[i][2], acc[i][2]));
                        acc[i][3] = fmaf(o1, X1, fmaf(s1, d[i][3], acc[i][3]));
                    }
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
    }
    (void)MB;

    // ---------------- cross-warp reduction + epilogue ----------------
    Acc *red = reinterpret_cast<Acc *>(smem + L.red);
#pragma unroll
    for (int i = 0; i < kSG; ++i)
#pragma unroll
        for (int e = 0; e < 4; ++e) red[((warp * kSG + i) * 32 + lane) * 4 + e] = acc[i][e];
    named_bar_sync(1, kNW * 32);

    const int tid = threadIdx.x;
    auto finalize = [&](const Acc *v, int r, int tok) {
        if (MODE == 0) {
#pragma unroll
            for (int i = 0; i < kSG; ++i) {
                const int row = strip[i] * kStripRows + r;
                if (!valid[i] || row >= p.N) continue;
                const GemvSrc &sr = p.src[0];
                float out;
                if (LAYOUT == kLayoutS8)
                    out = (float)v[i] * (sr.scale * p.sx[tok]);
                else
                    out = (float)v[i];
                if (sr.bias) out += sr.bias[row];
                if (sr.out_cols) {
                    float os = 0.0f;
#pragma unroll
                    for (int k = 0; k < 8; ++k) {
                        const int col = sr.out_cols[(size_t)row * 8 + k];
                        if (col >= 0) os += __half2float(sr.out_w[(size_t)row * 8 + k]) * p.xrow[(size_t)tok * p.K + col];
                    }
                    out += os;
                }
                float *yp = p.y + (size_t)tok * p.ldy + row;
                *yp = p.accumulate ? *yp + out : out;
            }
        } else {
            const int row = strip[0] * kStripRows + r;
            if (row >= p.N) return;
            float gv, uv;
            if (LAYOUT == kLayoutS8) {
                gv = (float)v[0] * (p.src[0].scale * p.sx[tok]);
                uv = (float)v[1] * (p.src[1].scale * p.sx[tok]);
            } else {
                gv = (float)v[0];
                uv = (float)v[1];
            }
            if (p.src[0].bias) gv += p.src[0].bias[row];
            if (p.src[1].bias) uv += p.src[1].bias[row];
            float *yp = p.y + (size_t)tok * p.ldy + row;
            *yp = silu_f(gv) * uv;
        }
    };

    Acc *ws = static_cast<Acc *>(p.ws);
    for (int q = tid; q < 128; q += kNW * 32) {
        const int r = q >> 3, tok = q & 7;
        if (tok >= M) continue;
        const int ln = (r & 7) * 4 + (tok >> 1), e = (r >> 3) * 2 + (tok & 1);
        Acc v[kSG];
#pragma unroll
        for (int i = 0; i < kSG; ++i) {
            Acc s = 0;
            for (int w = 0; w < kNW; ++w) s += red[((w * kSG + i) * 32 + ln) * 4 + e];
            v[i] = s;
        }
        if (p.n_ks == 1) {
            finalize(v, r, tok);
        } else {
#pragma unroll
            for (int i = 0; i < kSG; ++i) ws[((size_t)unit * kSG + i) * 128 + q] = v[i];
        }
    }
    if (p.n_ks > 1) {
        __threadfence();
        named_bar_sync(1, kNW * 32);
        if (tid == 0) {
            const unsigned old = atomicAdd(&p.counters[sg], 1u);
            *s_flag = (old == (unsigned)(p.n_ks - 1)) ? 1 : 0;
        }
        named_bar_sync(1, kNW * 32);
        if (*s_flag) {
            __threadfence();
            for (int q = tid; q < 128; q += kNW * 32) {
                const int r = q >> 3, tok = q & 7;
                if (tok >= M) continue;
                Acc v[kSG];
#pragma unroll
                for (int i = 0; i < kSG; ++i) {
                    Acc s = 0;
                    for (int k = 0; k < p.n_ks; ++k)
                        s += __ldcg(&ws[(((size_t)sg * p.n_ks + k) * kSG + i) * 128 + q]);
                    v[i] = s;
                }
                finalize(v, r, tok);
            }
            if (tid == 0) atomicExch(&p.counters[sg], 0u);
        }
    }
}

// ----------------------------------------------------------------------------
// host side: plan + launch
// ----------------------------------------------------------------------------

static int epilogue_cols(const DevMatrix &w) {
    if (w.layout == kLayoutS8) return 32;
    const int kc = chunk_cols(w.bits);
    const int grp = (w.n_groups == 1) ? kc : w.group;
    return std::min(grp, kc);
}

int plan_gemv(const DevMatrix &w, int M, int mode, bool xsplit, GemvPlan *plan) {
    GemvPlan P;
    P.mode = mode;
    P.sg = kSG;
    P.xsplit = xsplit;
    P.e_cols = epilogue_cols(w);
    const int kc = w.layout == kLayoutS8 ? 32 : chunk_cols(w.bits);
    const int steps = w.layout == kLayoutS8 ? 1 : kc / 16;
    const int ne = w.layout == kLayoutS8 ? 0 : kc / P.e_cols;
    P.n_sg = mode == 1 ? w.n_strips : ceil_div(w.n_strips, kSG);
    const size_t x_per_chunk = (size_t)steps * M * 32 * (xsplit ? 2 : 1) + (size_t)ne * 32;
    int cpk_max = (int)std::max<size_t>(1, kXMaxBytes / x_per_chunk);
    const int want_ks = std::max(1, ceil_div(kTargetUnits, P.n_sg));
    int cpk = ceil_div(w.n_chunks, want_ks);
    cpk = std::max(cpk, std::min(16, w.n_chunks));
    cpk = std::min(cpk, cpk_max);
    // keep the K-slice on a group boundary so each slice's metadata is whole groups
    if (w.layout == kLayoutF16 && w.n_groups > 1 && w.group > kc) {
        const int cpg = w.group / kc;
        cpk = std::max(cpg, cpk / cpg * cpg);
    }
    P.cpk = cpk;
    P.n_ks = ceil_div(w.n_chunks, cpk);
    if (w.layout == kLayoutF16) {
        if (w.n_groups == 1)
            P.gps = 1;
        else
            P.gps = ceil_div((long)cpk * kc, w.group) + 1;
    } else {
        P.gps = 0;
    }
    const SmemLayout L = smem_layout(w.layout, w.bits, cpk, M, xsplit, P.e_cols, P.gps, w.meta_kind);
    P.smem = L.total;
    P.xf_bytes = (size_t)w.n_chunks * steps * M * 32;
    P.xs_bytes = w.layout == kLayoutF16 ? (size_t)w.n_chunks * ne * 32 : 0;
    P.ws_bytes = P.n_ks > 1 ? (size_t)P.n_sg * P.n_ks * kSG * 128 * 4 : 0;
    P.counters = P.n_ks > 1 ? P.n_sg : 0;
    *plan = P;
    return 0;
}

template <int BITS, int LAYOUT, int E, bool XSPLIT, int MODE>
static cudaError_t launch_t(const GemvPlan &plan, const GemvParams &p, cudaStream_t st) {
    auto kern = gemv_kernel<BITS, LAYOUT, E, XSPLIT, MODE>;
    static bool attr_set = false;
    if (!attr_set) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        if (e != cudaSuccess) return e;
        attr_set = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(plan.n_sg * plan.n_ks));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = plan.smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, p);
}

template <int BITS, int LAYOUT, int E>
static cudaError_t launch_x(const GemvPlan &plan, const GemvParams &p, cudaStream_t st) {
    if (plan.mode == 0)
        return plan.xsplit ? launch_t<BITS, LAYOUT, E, true, 0>(plan, p, st)
                           : launch_t<BITS, LAYOUT, E, false, 0>(plan, p, st);
    return plan.xsplit ? launch_t<BITS, LAYOUT, E, true, 1>(plan, p, st)
                       : launch_t<BITS, LAYOUT, E, false, 1>(plan, p, st);
}

cudaError_t launch_gemv(const DevMatrix &w0, const DevMatrix *w1, const GemvPlan &plan, const GemvParams &p,
                        cudaStream_t st) {
    (void)w1;
    if (w0.layout == kLayoutS8) {
        if (plan.mode == 0) return launch_t<8, kLayoutS8, 32, false, 0>(plan, p, st);
        return launch_t<8, kLayoutS8, 32, false, 1>(plan, p, st);
    }
    switch (w0.bits) {
    case 8:
        return launch_x<8, kLayoutF16, 32>(plan, p, st);
    case 4:
        return launch_x<4, kLayoutF16, 64>(plan, p, st);
    case 2:
        if (plan.e_cols == 64) return launch_x<2, kLayoutF16, 64>(plan, p, st);
        return launch_x<2, kLayoutF16, 128>(plan, p, st);
    default:
        return cudaErrorInvalidValue;
    }
}

}  // namespace chpe
