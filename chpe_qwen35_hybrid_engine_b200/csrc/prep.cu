// prep.cu -- activation-fragment preparation, dynamic int8 activation
// quantization, weight repacking into the strip layout, and the GPU
// quantizers used to build device tensors from fp32 weights.
#include <cooperative_groups.h>

#include <algorithm>

#include "common.cuh"
#include "internal.h"
#include "xsrc.cuh"

namespace chpe {

// ---------------------------------------------------------------------------
// activations
// ---------------------------------------------------------------------------

// Activation fragments of the fp16 GEMV path.  One cluster of C CTAs
// (fill_ctas) per activation row tok = blockIdx.y; CTA c owns fragment units
// [u0, u1) (fill_range), kFillThreads of them at a time.  Unit u = 4 * s + t
// (k-step s, lane column t) holds columns 16s + 2t + {0, 1, 8, 9}; fragments
// are stored as 16-byte units so a consumer fetches two k-steps (or, for fp32
// input, the hi and lo parts of one k-step) with one load:
//   split (fp32 x):  unit (s, m, t) = {hi(16s+2t..), hi(16s+2t+8..), lo(..), lo(..)}
//   fp16/bf16 x:     unit (s/2, m, t) = {step 2u: ..., step 2u+1: ...}
// Pass 1 reads each source value once (kept in registers, with its RMSNorm
// gamma, for the first kFillCache units of a thread) and reduces the CTA's
// range: the sum of squares (RMSNorm, in the canonical order of xsrc.cuh) and
// the largest |value|.  Each CTA writes them into every peer's shared memory
// (distributed shared memory, one cluster barrier) and all combine them in
// range order, so the whole cluster agrees on the RMSNorm
// scale and on the row's power-of-two scale 2^e (row_scale_exp), which keeps
// every scaled value inside fp16's range; xe[tok] = 2^-e undoes it in the
// GEMV epilogue.  Pass 2 scales, splits and stores.
// `bits` selects the per-k-step power-of-two pre-scale that matches where the
// GEMV kernel reads the codes (unpack_f16): 4-bit odd k-steps of a chunk /16,
// 2-bit k-step j of a chunk / 4^(j%4), 8-bit none.  The sum of each E-column
// block (what the zero-point term multiplies) is taken over the values the
// MMA sees, with the k-step pre-scale undone, from the E/4 consecutive threads
// that hold the block.
constexpr int kFillCache = 4;  // units per thread held in registers between the passes

// The tensor-parallel all-reduce fused in front of a fill (FillExchange), on
// this CTA's columns of row tok, leaving the new hidden values in the
// thread's register cache: the exchange of comm.cu (tagged words, one NVLink
// trip), then hidden += (sum of the ranks' partials in rank order) -- the
// one-shot all-reduce's arithmetic -- and the last CTA of the launch advances
// the epoch.  A thread whose wait runs out (1 s for all its words) marks the
// comm object failed; the CTA then leaves hidden as it was and still takes
// part in the fill's cluster barrier, so no CTA is left waiting.
__device__ __forceinline__ void fill_exchange(const FillExchange &ex, int tok, int K, int u0, int u1,
                                              float (&cv)[kFillCache][4]) {
    __shared__ int s_ok;
    const int tid = threadIdx.x;
    const bool failed = *reinterpret_cast<const volatile unsigned *>(&ex.ctr[2]) != 0u;
    const unsigned epoch = *reinterpret_cast<const volatile unsigned *>(&ex.ctr[0]) + 1u;
    const size_t base = (size_t)tok * K;
    const size_t slot = ((size_t)(epoch & 1u) * ex.world + ex.rank) * ex.slot_elems + base;
    if (tid == 0) s_ok = failed ? 0 : 1;
#pragma unroll
    for (int i = 0; i < kFillCache; ++i) {
        const int u = u0 + tid + i * kFillThreads;
        int kk[4];
        unit_cols(u, kk);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const bool in = u < u1 && kk[q] < K;
            const float p = in ? ex.part[base + kk[q]] : 0.0f;
            cv[i][q] = p;
            if (in && !failed && !ex.pushed)
                for (int r = 0; r < ex.world; ++r)
                    if (r != ex.rank) st_tagged(ex.peers.tagged[r] + slot + kk[q], p, epoch);
        }
    }
    if (failed && tid == 0) atomicExch(ex.err, kErrCommFailed);
    const unsigned long long *own = ex.peers.tagged[ex.rank] + (size_t)(epoch & 1u) * ex.world * ex.slot_elems + base;
    bool ok = !failed;
    const unsigned long long t0 = global_timer_ns();
#pragma unroll
    for (int i = 0; i < kFillCache; ++i) {
        const int u = u0 + tid + i * kFillThreads;
        if (u >= u1) continue;
        int kk[4];
        unit_cols(u, kk);
        size_t idx[4];
        bool valid[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            idx[q] = (size_t)kk[q];
            valid[q] = kk[q] < K;
        }
        // the ranks' sums of the unit's four columns; hidden is added below
        sum_tagged<4>(own, ex.slot_elems, idx, valid, ex.world, ex.rank, cv[i], epoch, t0, ok, cv[i]);
    }
    if (!ok && !failed) {
        atomicExch(ex.err, kErrCommWait);
        atomicExch(&ex.ctr[2], 1u);  // failed: no later exchange on this object until a reset
        *reinterpret_cast<volatile unsigned *>(ex.host_failed) = 1u;
        s_ok = 0;
    }
    __syncthreads();
    const bool all_ok = s_ok != 0;
#pragma unroll
    for (int i = 0; i < kFillCache; ++i) {
        const int u = u0 + tid + i * kFillThreads;
        int kk[4];
        unit_cols(u, kk);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            if (u < u1 && kk[q] < K) {
                float h = ex.hidden[base + kk[q]];
                if (all_ok) {
                    h += cv[i][q];
                    ex.hidden[base + kk[q]] = h;
                }
                cv[i][q] = h;
            }
        }
    }
    if (tid == 0) {
        __threadfence();
        if (atomicAdd(&ex.ctr[1], 1u) == gridDim.x * gridDim.y - 1) {
            ex.ctr[1] = 0u;
            if (!atomicAdd(&ex.ctr[2], 0u)) ex.ctr[0] = epoch;
        }
    }
}

template <bool EXCH>  // with the fused all-reduce (ex), or without (ex unused)
__global__ void __launch_bounds__(kFillThreads) chpe_xfill_f16_kernel(const XSrc s, int M, int K, int Kp, int E,
                                                                     int split, int bits, uint2 *__restrict__ xf,
                                                                     float *__restrict__ xs, float *__restrict__ xe,
                                                                     const FillExchange ex) {
    namespace cg = cooperative_groups;
    cg::cluster_group cluster = cg::this_cluster();
    __shared__ float red[2 * kFillWarps];
    __shared__ float2 stats[kFillMaxCtas];  // (sum of squares, largest |value|) of every CTA of the row's cluster
    grid_dependents_launch();
    const int tok = blockIdx.y;
    const int nunits = Kp / 4;
    const int C = (int)cluster.num_blocks();
    const int c = (int)cluster.block_rank();
    int u0, u1;
    fill_range(nunits, C, c, u0, u1);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const bool rms = s.op == kXRmsnorm;
    const float *xrow = static_cast<const float *>(s.x) + (size_t)tok * s.ldx;
    // source value of column k: raw x for RMSNorm (normalised in pass 2), else the op's value
    auto src = [&](int k) -> float {
        if (k >= K) return 0.0f;
        return rms ? xrow[k] : xsrc_value(s, tok, k, 1.0f);
    };
    float cv[kFillCache][4], cg4[kFillCache][4];  // cached values (and RMSNorm gammas)
    // RMSNorm's gamma is a weight, not the upstream kernel's output: its loads
    // go out before the wait for the upstream grid
    if (rms) {
#pragma unroll
        for (int i = 0; i < kFillCache; ++i) {
            const int u = u0 + tid + i * kFillThreads;
            int kk[4];
            unit_cols(u, kk);
#pragma unroll
            for (int q = 0; q < 4; ++q) cg4[i][q] = (u < u1 && kk[q] < K) ? s.aux[kk[q]] : 0.0f;
        }
    }
    grid_dependency_wait();
    // with an exchange, the cache already holds the new hidden values (every
    // unit of the CTA fits the cache: xfill_exchange_fits)
    constexpr bool exch = EXCH;
    if constexpr (EXCH) fill_exchange(ex, tok, K, u0, u1, cv);
    float ss = 0.0f, am = 0.0f;
#pragma unroll
    for (int i = 0; i < kFillCache; ++i) {
        const int u = u0 + tid + i * kFillThreads;
        if (u < u1) {
            int kk[4];
            unit_cols(u, kk);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const float v = exch ? cv[i][q] : src(kk[q]);
                cv[i][q] = v;
                if (rms) {
                    const float g = cg4[i][q];
                    ss = fmaf(v, v, ss);
                    am = fmaxf(am, fabsf(__fmul_rn(v, g)));
                } else {
                    am = fmaxf(am, fabsf(v));
                }
            }
        }
    }
    for (int u = u0 + tid + kFillCache * kFillThreads; u < u1; u += kFillThreads) {  // units past the cache
        int kk[4];
        unit_cols(u, kk);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const float v = src(kk[q]);
            if (rms) {
                ss = fmaf(v, v, ss);
                am = fmaxf(am, fabsf(__fmul_rn(v, kk[q] < K ? s.aux[kk[q]] : 0.0f)));
            } else {
                am = fmaxf(am, fabsf(v));
            }
        }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        ss += __shfl_xor_sync(0xffffffffu, ss, off);
        am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, off));
    }
    if (lane == 0) {
        red[warp] = ss;
        red[kFillWarps + warp] = am;
    }
    __syncthreads();
    // thread r < C writes this CTA's statistics into slot c of CTA r (distributed
    // shared memory); one cluster barrier later every CTA holds all of them
    if (tid < C) {
        float t = 0.0f, m = 0.0f;
#pragma unroll
        for (int w = 0; w < kFillWarps; ++w) {
            t += red[w];
            m = fmaxf(m, red[kFillWarps + w]);
        }
        *cluster.map_shared_rank(&stats[c], tid) = make_float2(t, m);
    }
    cluster.sync();
    float tot = 0.0f, amax = 0.0f;
    for (int r = 0; r < C; ++r) {
        const float2 v = stats[r];
        tot += v.x;
        amax = fmaxf(amax, v.y);
    }
    const float inv = rms ? inv_rms_of(tot, K, s.eps) : 1.0f;
    const int e = row_scale_exp(rms ? amax * inv : amax);
    if (c == 0 && tid == 0) xe[tok] = pow2_of(-e);
    const int steps = (256 / bits) / 16;  // k-steps per chunk
    for (int i = 0; u0 + i * kFillThreads < u1; ++i) {
        const int u = u0 + tid + i * kFillThreads;
        float part = 0.0f;
        if (u < u1) {
            const int st = u >> 2, t = u & 3;
            const int j = st % steps;
            const int sh = bits == 4 ? 4 * (j & 1) : bits == 2 ? 2 * (j & 3) : 0;
            const float down = pow2_of(e - sh), up = pow2_of(sh);
            int kk[4];
            unit_cols(u, kk);
            float v4[4], g4[4];
            if (i < kFillCache) {
#pragma unroll
                for (int ci = 0; ci < kFillCache; ++ci)
                    if (ci == i) {
#pragma unroll
                        for (int q = 0; q < 4; ++q) {
                            v4[q] = cv[ci][q];
                            g4[q] = cg4[ci][q];
                        }
                    }
            } else {
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    v4[q] = src(kk[q]);
                    g4[q] = rms && kk[q] < K ? s.aux[kk[q]] : 0.0f;
                }
            }
            __half h[4], l[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                float v = v4[q];
                if (rms) v = __fmul_rn(__fmul_rn(v, inv), g4[q]);
                v *= down;
                h[q] = __float2half_rn(v);
                l[q] = split ? __float2half_rn(v - __half2float(h[q])) : __float2half_rn(0.0f);
                part += (__half2float(h[q]) + __half2float(l[q])) * up;
            }
            const uint2 hv = make_uint2(pack_h2(h[0], h[1]), pack_h2(h[2], h[3]));
            if (split) {
                const size_t v = ((size_t)st * M + tok) * 4 + t;
                xf[2 * v] = hv;
                xf[2 * v + 1] = make_uint2(pack_h2(l[0], l[1]), pack_h2(l[2], l[3]));
            } else {
                const size_t v = ((size_t)(st >> 1) * M + tok) * 4 + t;
                xf[2 * v + (st & 1)] = hv;
            }
        }
        // E/4 consecutive threads (8, 16 or 32, aligned) hold one E-column
        // block; ranges are whole 32-unit groups, so a warp is all in or all out
        if (u0 + i * kFillThreads + 32 * warp < u1) {
            for (int off = E / 8; off > 0; off >>= 1) part += __shfl_xor_sync(0xffffffffu, part, off);
            if (u < u1 && (u % (E / 4)) == 0) xs[(size_t)(u / (E / 4)) * 8 + tok] = part;
        }
    }
}

bool xfill_exchange_fits(int M, int Kp) {
    (void)M;
    const int nunits = Kp / 4, C = fill_ctas(nunits);
    int most = 0;
    for (int c = 0; c < C; ++c) {
        int u0, u1;
        fill_range(nunits, C, c, u0, u1);
        most = std::max(most, u1 - u0);
    }
    return most <= kFillCache * kFillThreads;
}

cudaError_t launch_xfill_f16(const XSrc &s, int M, int K, int Kp, int e_cols, bool xsplit, int bits, void *xf,
                             float *xs, float *xe, cudaStream_t st, const FillExchange *ex) {
    const int C = fill_ctas(Kp / 4);
    if (ex && ex->world > 0)
        return launch_pdl_cluster(chpe_xfill_f16_kernel<true>, dim3(C, M), dim3(kFillThreads), (unsigned)C, 0, st, s,
                                  M, K, Kp, e_cols, xsplit ? 1 : 0, bits, static_cast<uint2 *>(xf), xs, xe, *ex);
    const FillExchange none{};
    return launch_pdl_cluster(chpe_xfill_f16_kernel<false>, dim3(C, M), dim3(kFillThreads), (unsigned)C, 0, st, s, M,
                              K, Kp, e_cols, xsplit ? 1 : 0, bits, static_cast<uint2 *>(xf), xs, xe, none);
}

cudaError_t launch_xprep_f16(const void *x, int x_dtype, int M, int K, int Kp, int e_cols, bool xsplit, int bits,
                             void *xf, float *xs, float *xe, cudaStream_t st) {
    XSrc s;
    s.op = kXPlain;
    s.x = x;
    s.dt = x_dtype;
    s.ldx = K;
    return launch_xfill_f16(s, M, K, Kp, e_cols, xsplit, bits, xf, xs, xe, st);
}

// The source op's values as fp32 rows [M][K], for the int8 (W8A8) path, which
// quantizes them per row exactly as the reference does, and for the outlier
// columns' fp32 activations.  RMSNorm statistics in the reference's own order
// (ref_order_inv_rms), so the int8 codes match the reference's bit for bit.
__global__ void __launch_bounds__(256) chpe_xmaterialize_kernel(const XSrc s, int K, float *__restrict__ out) {
    __shared__ float s_inv;
    pdl_begin();
    const int tok = blockIdx.y;
    if (threadIdx.x < 32) {
        const float v = s.op == kXRmsnorm ? ref_order_inv_rms(static_cast<const float *>(s.x) + (size_t)tok * s.ldx,
                                                               K, s.eps)
                                          : 1.0f;
        if (threadIdx.x == 0) s_inv = v;
    }
    __syncthreads();
    const float inv = s_inv;
    for (int k = blockIdx.x * blockDim.x + threadIdx.x; k < K; k += gridDim.x * blockDim.x)
        out[(size_t)tok * K + k] = xsrc_value(s, tok, k, inv);
}

cudaError_t launch_xmaterialize(const XSrc &s, int M, int K, int Kp, float *out, cudaStream_t st) {
    (void)Kp;
    const int gx = std::min(32, (K + 255) / 256);
    return launch_pdl(chpe_xmaterialize_kernel, dim3(gx, M), dim3(256), 0, st, s, K, out);
}

__device__ __forceinline__ uint32_t pack4_i8(const int8_t *p, int k, int K) {
    uint32_t w = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint32_t b = (k + i < K) ? (uint32_t)(uint8_t)p[k + i] : 0u;
        w |= b << (8 * i);
    }
    return w;
}

// int8 activations [M][K] -> fragments [kstep32][M][4] uint2.
__global__ void chpe_xprep_s8_kernel(const int8_t *__restrict__ xq, int M, int K, int nsteps, uint2 *__restrict__ xf) {
    pdl_begin();
    const size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    const size_t total = (size_t)nsteps * M * 4;
    if (idx >= total) return;
    const int t = (int)(idx & 3);
    const int tok = (int)((idx >> 2) % M);
    const int s = (int)(idx / (4 * (size_t)M));
    const int8_t *row = xq + (size_t)tok * K;
    const int kb = 32 * s + 4 * t;
    xf[idx] = make_uint2(pack4_i8(row, kb, K), pack4_i8(row, kb + 16, K));
}

cudaError_t launch_xprep_s8(const int8_t *xq, int M, int K, int Kp, void *xf, cudaStream_t st) {
    const int nsteps = Kp / 32;
    const size_t total = (size_t)nsteps * M * 4;
    return launch_pdl(chpe_xprep_s8_kernel, dim3((unsigned)((total + 255) / 256)), dim3(256), 0, st, xq, M, K, nsteps,
                      static_cast<uint2 *>(xf));
}

// Per-row dynamic int8 quantization, bit-exact with the reference
// (src/kernels/neon.zig:644-670): s = max|x|/127 (1 when max <= 1e-9),
// q = clamp(round_half_away(x * (1/s)), -128, 127).  One block per row.
__global__ void chpe_act_quant_s8_kernel(const float *__restrict__ x, int M, int K, int nsteps, int8_t *__restrict__ q,
                                    float *__restrict__ scales, uint2 *__restrict__ xf) {
    __shared__ float red[32];
    __shared__ float s_inv;
    pdl_begin();
    const int tok = blockIdx.x;
    const float *row = x + (size_t)tok * K;
    float m = 0.0f;
    for (int k = threadIdx.x; k < K; k += blockDim.x) m = fmaxf(m, fabsf(row[k]));
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x == 0) {
        float mm = 0.0f;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) mm = fmaxf(mm, red[w]);
        const float scale = (mm > 1e-9f) ? __fdiv_rn(mm, 127.0f) : 1.0f;
        s_inv = __fdiv_rn(1.0f, scale);
        if (scales) scales[tok] = scale;
    }
    __syncthreads();
    const float inv = s_inv;
    auto quant = [&](int k) -> uint32_t {
        if (k >= K) return 0u;
        const float r = roundf(__fmul_rn(row[k], inv));
        const float c = fmaxf(-128.0f, fminf(127.0f, r));
        return (uint32_t)(uint8_t)(int8_t)c;
    };
    if (q)
        for (int k = threadIdx.x; k < K; k += blockDim.x) q[(size_t)tok * K + k] = (int8_t)(uint8_t)quant(k);
    if (xf) {
        for (int e = threadIdx.x; e < nsteps * 4; e += blockDim.x) {
            const int s = e >> 2, t = e & 3;
            const int kb = 32 * s + 4 * t;
            uint32_t w0 = 0, w1 = 0;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                w0 |= quant(kb + i) << (8 * i);
                w1 |= quant(kb + 16 + i) << (8 * i);
            }
            xf[((size_t)s * M + tok) * 4 + t] = make_uint2(w0, w1);
        }
    }
}

cudaError_t launch_act_quant_s8(const float *x, int M, int K, int Kp, int8_t *q, float *scales, void *xf,
                                cudaStream_t st) {
    return launch_pdl(chpe_act_quant_s8_kernel, dim3(M), dim3(256), 0, st, x, M, K, Kp / 32, q, scales,
                      static_cast<uint2 *>(xf));
}

// ---------------------------------------------------------------------------
// weights
// ---------------------------------------------------------------------------

// Code of element (row, k) from packed row-major codes of `sbits` bits each
// (LSB first within a byte); 0 outside the matrix (padding).
__device__ __forceinline__ uint32_t src_code(const uint8_t *src, size_t stride, int N, int K, int sbits, int row,
                                             int k, uint32_t xorv) {
    if (row >= N || k >= K) return 0u;
    const size_t bit = (size_t)k * sbits;
    const uint32_t byte = src[(size_t)row * stride + (bit >> 3)];
    const uint32_t mask = (1u << sbits) - 1u;
    return ((byte >> (bit & 7)) & mask) ^ xorv;
}

// One thread per 32-bit word of the code area of the strip layout.
__global__ void chpe_repack_codes_kernel(const uint8_t *__restrict__ src, size_t stride, int N, int K, int sbits, int bits,
                                    int layout, uint32_t xorv, uint8_t *__restrict__ dst, int n_strips,
                                    int n_blocks, int block_bytes) {
    const size_t wi = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int n_chunks = n_blocks * kChunksPerBlock;
    const size_t total = (size_t)n_strips * n_chunks * 128;
    if (wi >= total) return;
    const int lw = (int)(wi & 127);
    const size_t sc = wi >> 7;
    const int chunk = (int)(sc % n_chunks);
    const int strip = (int)(sc / n_chunks);
    const int lane = lw >> 2, r = lw & 3;
    const int g = lane >> 2, t = lane & 3;
    const int row = strip * kStripRows + g + 8 * (r & 1);
    uint32_t w = 0;
    if (layout == kLayoutS8) {
        const int kb = chunk * 32 + 4 * t + 16 * (r >> 1);
#pragma unroll
        for (int i = 0; i < 4; ++i) w |= src_code(src, stride, N, K, sbits, row, kb + i, 0u) << (8 * i);
    } else {
        const int kc = 256 / bits;
        const int col = 2 * t + 8 * (r >> 1);
        const int kb = chunk * kc + col;
        if (bits == 4) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                w |= src_code(src, stride, N, K, sbits, row, kb + 16 * j, xorv) << (4 * j);
                w |= src_code(src, stride, N, K, sbits, row, kb + 16 * j + 1, xorv) << (4 * (j + 4));
            }
        } else if (bits == 2) {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                w |= src_code(src, stride, N, K, sbits, row, kb + 16 * j, xorv) << (2 * j);
                w |= src_code(src, stride, N, K, sbits, row, kb + 16 * j + 1, xorv) << (2 * (j + 8));
            }
        } else {
            w |= src_code(src, stride, N, K, sbits, row, kb, xorv);
            w |= src_code(src, stride, N, K, sbits, row, kb + 1, xorv) << 8;
            w |= src_code(src, stride, N, K, sbits, row, kb + 16, xorv) << 16;
            w |= src_code(src, stride, N, K, sbits, row, kb + 17, xorv) << 24;
        }
    }
    const int blk = chunk / kChunksPerBlock, cib = chunk % kChunksPerBlock;
    const size_t off = ((size_t)strip * n_blocks + blk) * block_bytes + (size_t)cib * kChunkBytes + (size_t)lw * 4;
    *reinterpret_cast<uint32_t *>(dst + off) = w;
}

cudaError_t launch_repack_codes(const uint8_t *src, size_t row_stride, int src_bits, uint32_t xorv,
                                const DevMatrix &m, cudaStream_t st) {
    const size_t total = (size_t)m.n_strips * m.n_blocks * kChunksPerBlock * 128;
    note_launch();
    chpe_repack_codes_kernel<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(src, row_stride, m.N, m.K, src_bits, m.bits,
                                                                        m.layout, xorv, m.codes, m.n_strips,
                                                                        m.n_blocks, m.block_bytes);
    return cudaGetLastError();
}

// One thread per metadata entry (strip, block, group-in-block, row).  The
// group of entry gib of block b is b*span/group + gib; groups past the matrix
// (K padding) and rows past N get zero entries.
__global__ void chpe_meta_repack_kernel(int kind, const __half *__restrict__ s, const __half *__restrict__ z,
                                   const float *__restrict__ fs, const float *__restrict__ fo, float zc, int N,
                                   int n_groups, int group, int span, int gpb, int n_strips, int n_blocks,
                                   int block_bytes, uint8_t *__restrict__ dst) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    const size_t total = (size_t)n_strips * n_blocks * gpb * 16;
    if (i >= total) return;
    const int r16 = (int)(i & 15);
    size_t rest = i >> 4;
    const int gib = (int)(rest % gpb);
    rest /= gpb;
    const int blk = (int)(rest % n_blocks);
    const int strip = (int)(rest / n_blocks);
    const int row = strip * kStripRows + r16;
    const long grp = (long)blk * span / group + gib;
    const bool in = row < N && grp < n_groups;
    uint8_t *base = dst + ((size_t)strip * n_blocks + blk) * block_bytes + kBlockCodeBytes;
    const int e = gib * 16 + (r16 & 7) * 2 + (r16 >> 3);  // rows g and g+8 side by side
    if (kind == kMetaS16) {
        reinterpret_cast<__half *>(base)[e] = in ? s[(size_t)row * n_groups + grp] : __float2half_rn(0.0f);
    } else if (kind == kMetaSZ16) {
        reinterpret_cast<__half2 *>(base)[e] =
            in ? __halves2half2(s[(size_t)row * n_groups + grp], z[(size_t)row * n_groups + grp])
               : __halves2half2(__float2half_rn(0.0f), __float2half_rn(0.0f));
    } else {
        float2 v = make_float2(0.0f, 0.0f);
        if (in) {
            const float sc = fs[row];
            // offset per unit of x, times 2^-24 (the GEMV scales its sums by 2^24 at the end)
            v = make_float2(sc, ((fo ? fo[row] : 0.0f) - zc * sc) * (1.0f / 16777216.0f));
        }
        reinterpret_cast<float2 *>(base)[e] = v;
    }
}

cudaError_t launch_meta_repack(const __half *s, const __half *z, const float *fs, const float *fo,
                               float zc_for_f32, const DevMatrix &m, cudaStream_t st) {
    const size_t total = (size_t)m.n_strips * m.n_blocks * m.gpb * 16;
    note_launch();
    chpe_meta_repack_kernel<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(
        m.meta_kind, s, z, fs, fo, zc_for_f32, m.N, m.n_groups, m.group, m.span, m.gpb, m.n_strips, m.n_blocks,
        m.block_bytes, m.codes);
    return cudaGetLastError();
}

// GPU grouped quantizers (the formulas of chpe_quantize_group_dev in the header):
// one warp per (row, group); codes are written one byte per weight.
__global__ void chpe_quant_group_kernel(const float *__restrict__ w, int N, int K, int group, int bits, int symmetric,
                                   uint8_t *__restrict__ codes, __half *__restrict__ scales,
                                   __half *__restrict__ zeros) {
    const size_t gw = ((size_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    const int G = K / group;
    if (gw >= (size_t)N * G) return;
    const int row = (int)(gw / G), grp = (int)(gw % G);
    const float *v = w + (size_t)row * K + (size_t)grp * group;
    float mn = INFINITY, mx = -INFINITY, am = 0.0f;
    for (int i = lane; i < group; i += 32) {
        mn = fminf(mn, v[i]);
        mx = fmaxf(mx, v[i]);
        am = fmaxf(am, fabsf(v[i]));
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, off));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
        am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, off));
    }
    if (symmetric) {
        __half s = __float2half_rn(am > 1e-8f ? __fdiv_rn(am, 127.0f) : 1.0f);
        float s32 = __half2float(s);
        if (!(s32 > 0.0f)) {
            s32 = 1.0f;
            s = __float2half_rn(1.0f);
        }
        for (int i = lane; i < group; i += 32) {
            const float q = fminf(fmaxf(rintf(__fdiv_rn(v[i], s32)), -127.0f), 127.0f);
            codes[(size_t)row * K + (size_t)grp * group + i] = (uint8_t)(int8_t)q;
        }
        if (lane == 0) scales[(size_t)row * G + grp] = s;
    } else {
        const float qmax = (float)((1 << bits) - 1);
        const float range = mx - mn;
        __half s = __float2half_rn(range > 1e-8f ? __fdiv_rn(range, qmax) : 1.0f);
        float s32 = __half2float(s);
        if (!(s32 > 0.0f)) {
            s32 = 1.0f;
            s = __float2half_rn(1.0f);
        }
        const float zf = fminf(fmaxf(rintf(__fdiv_rn(-mn, s32)), 0.0f), qmax);
        for (int i = lane; i < group; i += 32) {
            const float c = fminf(fmaxf(rintf(__fdiv_rn(v[i], s32)) + zf, 0.0f), qmax);
            codes[(size_t)row * K + (size_t)grp * group + i] = (uint8_t)c;
        }
        if (lane == 0) {
            scales[(size_t)row * G + grp] = s;
            zeros[(size_t)row * G + grp] = __float2half_rn(zf);
        }
    }
}

cudaError_t launch_quant_group(const float *w, int N, int K, int group, int bits, int symmetric, uint8_t *codes,
                               __half *scales, __half *zeros, cudaStream_t st) {
    const size_t warps = (size_t)N * (K / group);
    const size_t threads = warps * 32;
    note_launch();
    chpe_quant_group_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, st>>>(w, N, K, group, bits, symmetric, codes,
                                                                        scales, zeros);
    return cudaGetLastError();
}

}  // namespace chpe

namespace chpe {

// ---------------------------------------------------------------------------
// read-back (the inverse of the repack): the strip layout -> row-major codes
// ---------------------------------------------------------------------------

// Code of element (row, k) as stored in the strip layout (layout.h), with the
// stored XOR undone: the code the matrix was uploaded with.
__device__ __forceinline__ uint32_t strip_code(const DevMatrix &m, int row, int k, uint32_t xorv) {
    const int strip = row / kStripRows, r16 = row % kStripRows;
    const int g = r16 & 7, hi = r16 >> 3;
    const int blk = k / m.span, kin = k % m.span;
    const int kc = 256 / m.bits;  // columns per chunk
    const int cib = kin / kc, cc = kin % kc;
    const uint8_t *chunk =
        m.codes + ((size_t)strip * m.n_blocks + blk) * m.block_bytes + (size_t)cib * kChunkBytes;
    if (m.layout == kLayoutS8) {
        const int rhi = cc / 16, t = (cc % 16) / 4, i = cc % 4;
        const int lw = (4 * g + t) * 4 + hi + 2 * rhi;
        return chunk[(size_t)lw * 4 + i];
    }
    const int j = cc / 16, c16 = cc % 16;
    const int rhi = c16 / 8, t = (c16 % 8) / 2, odd = c16 & 1;
    const int lw = (4 * g + t) * 4 + hi + 2 * rhi;
    const uint32_t w = reinterpret_cast<const uint32_t *>(chunk)[lw];
    uint32_t c;
    if (m.bits == 4)
        c = (w >> (4 * (j + 4 * odd))) & 0xFu;
    else if (m.bits == 2)
        c = (w >> (2 * (j + 8 * odd))) & 0x3u;
    else
        c = (w >> (8 * (2 * j + odd))) & 0xFFu;
    return c ^ xorv;
}

// One thread per output byte of the row-major packed codes (LSB first).
__global__ void chpe_unpack_codes_kernel(const DevMatrix m, uint32_t xorv, size_t row_bytes, uint8_t *__restrict__ out) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (size_t)m.N * row_bytes) return;
    const int row = (int)(i / row_bytes);
    const int byte = (int)(i % row_bytes);
    const int per = 8 / m.bits;
    uint32_t v = 0;
    for (int q = 0; q < per; ++q) {
        const int k = byte * per + q;
        if (k < m.K) v |= strip_code(m, row, k, xorv) << (m.bits * q);
    }
    out[i] = (uint8_t)v;
}

// One thread per (row, group): the fp16 scale (and zero) of the group, or the
// fp32 per-row scale of kMetaF32.
__global__ void chpe_unpack_meta_kernel(const DevMatrix m, __half *__restrict__ s, __half *__restrict__ z,
                                        float *__restrict__ fs) {
    const size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int ng = m.meta_kind == kMetaF32 ? 1 : m.n_groups;
    if (i >= (size_t)m.N * ng) return;
    const int row = (int)(i / ng), grp = (int)(i % ng);
    const int strip = row / kStripRows, r16 = row % kStripRows;
    const long k0 = (long)grp * (m.meta_kind == kMetaF32 ? m.K : m.group);
    const int blk = (int)(k0 / m.span);
    const int gib = m.gpb > 1 ? (int)((k0 % m.span) / m.group) : 0;
    const uint8_t *base = m.codes + ((size_t)strip * m.n_blocks + blk) * m.block_bytes + kBlockCodeBytes;
    const int e = gib * 16 + (r16 & 7) * 2 + (r16 >> 3);
    if (m.meta_kind == kMetaS16) {
        s[i] = reinterpret_cast<const __half *>(base)[e];
    } else if (m.meta_kind == kMetaSZ16) {
        const __half2 v = reinterpret_cast<const __half2 *>(base)[e];
        s[i] = __low2half(v);
        if (z) z[i] = __high2half(v);
    } else if (m.meta_kind == kMetaF32) {
        fs[i] = reinterpret_cast<const float2 *>(base)[e].x;
    }
}

cudaError_t launch_unpack(const DevMatrix &m, uint32_t xorv, size_t row_bytes, uint8_t *codes, __half *s, __half *z,
                          float *fs, cudaStream_t st) {
    const size_t n = (size_t)m.N * row_bytes;
    note_launch();
    chpe_unpack_codes_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(m, xorv, row_bytes, codes);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess || m.meta_kind == kMetaNone || (!s && !fs)) return e;
    const size_t nm = (size_t)m.N * (m.meta_kind == kMetaF32 ? 1 : m.n_groups);
    note_launch();
    chpe_unpack_meta_kernel<<<(unsigned)((nm + 255) / 256), 256, 0, st>>>(m, s, z, fs);
    return cudaGetLastError();
}

}  // namespace chpe
