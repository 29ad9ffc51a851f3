// xsrc.cuh -- device side of the activation sources (XSrc): the value of one
// activation as produced by a step's elementwise producer, shared by the
// fragment fill kernels (prep.cu) and the GEMV kernel's fused fill.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "common.cuh"
#include "internal.h"

namespace chpe {

__device__ __forceinline__ float load_x(const void *x, int dt, size_t i) {
    if (dt == 0) return static_cast<const float *>(x)[i];
    if (dt == 1) return __bfloat162float(static_cast<const __nv_bfloat16 *>(x)[i]);
    return __half2float(static_cast<const __half *>(x)[i]);
}

__device__ __forceinline__ uint32_t pack_h2(__half a, __half b) {
    __half2 h = __halves2half2(a, b);
    return *reinterpret_cast<uint32_t *>(&h);
}

// Value k of activation row tok, as produced by the source op (XSrc):
//   kXPlain     x[tok][k] (fp32 / bf16 / fp16)
//   kXRmsnorm   x[tok][k] * inv_rms(tok) * gamma[k]      (src/kernels/neon.zig:673-702)
//   kXSiluMul   silu(x[tok][k]) * aux[tok][k]            (src/kernels/neon.zig:705-712)
//   kXAttnStub  x[tok][src(k)]: the attention stand-in of src/engine.zig:619-623
//               (src = k % kv_dim), or head-aligned (query head h takes kv head h / group)
//   kXSsmStub   the Gated-DeltaNet stand-in, q = x[tok][k % qkv_dim], z = aux[tok][k]:
//               q * silu(z) (batch 1, src/engine.zig:651-654) or silu(q) * z (:813, :988)
__device__ __forceinline__ float xsrc_value(const XSrc &s, int tok, int k, float inv) {
    switch (s.op) {
    case kXRmsnorm: {
        const float v = static_cast<const float *>(s.x)[(size_t)tok * s.ldx + k];
        return __fmul_rn(__fmul_rn(v, inv), s.aux[k]);
    }
    case kXSiluMul:
        return silu_f(static_cast<const float *>(s.x)[(size_t)tok * s.ldx + k]) * s.aux[(size_t)tok * s.ld_aux + k];
    case kXAttnStub: {
        const int src = s.head_dim ? ((k / s.head_dim) / s.group) * s.head_dim + (k % s.head_dim) : (k % s.kv_dim);
        return static_cast<const float *>(s.x)[(size_t)tok * s.ldx + src];
    }
    case kXSsmStub: {
        const float q = static_cast<const float *>(s.x)[(size_t)tok * s.ldx + (k % s.qkv_dim)];
        const float z = s.aux[(size_t)tok * s.ld_aux + k];
        return s.silu_on_qkv ? silu_f(q) * z : q * silu_f(z);
    }
    default:
        return load_x(s.x, s.dt, (size_t)tok * s.ldx + k);
    }
}

// Partial sum of squares of one fp32 row for thread `tid` of `nthreads`:
// float4 j = tid, tid + nthreads, ... in order (each float4 in element order),
// then the tail past the last whole float4.  A fixed order, so every block
// that runs it with the same thread count gets the same bits.
__device__ __forceinline__ float row_sumsq_part(const float *row, int K, int tid, int nthreads) {
    float acc = 0.0f;
    const bool vec = (reinterpret_cast<uintptr_t>(row) & 15) == 0;
    const int K4 = vec ? K / 4 : 0;
    const float4 *r4 = reinterpret_cast<const float4 *>(row);
#pragma unroll 8
    for (int j = tid; j < K4; j += nthreads) {
        const float4 v = r4[j];
        acc = fmaf(v.x, v.x, acc);
        acc = fmaf(v.y, v.y, acc);
        acc = fmaf(v.z, v.z, acc);
        acc = fmaf(v.w, v.w, acc);
    }
    for (int k = 4 * K4 + tid; k < K; k += nthreads) acc = fmaf(row[k], row[k], acc);
    return acc;
}

// 1 / sqrt(mean + eps) from a total sum of squares (the rmsnorm scale).
__device__ __forceinline__ float inv_rms_of(float total, int K, float eps) {
    return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(total, (float)K), eps)));
}

// ---------------------------------------------------------------------------
// Row statistics of a fragment fill.  A row of Kp / 4 fragment units (unit u
// = columns 16(u/4) + 2(u%4) + {0, 1, 8, 9}) is cut into C = fill_ctas(units)
// contiguous ranges of whole 32-unit groups, one per CTA of a fill cluster of
// kFillThreads threads.  The RMSNorm sum of squares is defined in that
// CTA's order: thread t sums (fmaf) the squares of its units u0 + t,
// u0 + t + kFillThreads, ... element by element, a shuffle tree sums each
// warp, the warp partials are added in warp order, and the ranges' partials
// in range order.  block_row_stats computes the same bits in one block of 256
// or 512 threads (a 256-thread block plays two threads of the 512), so the
// fill kernel and the GEMV's fused fill agree.
// ---------------------------------------------------------------------------
constexpr int kFillThreads = 512;
constexpr int kFillMaxCtas = 8;  // a portable cluster
constexpr int kFillWarps = kFillThreads / 32;

__host__ __device__ inline int fill_ctas(int nunits) {
    const int c = (nunits + kFillThreads - 1) / kFillThreads;
    return c < 1 ? 1 : (c > kFillMaxCtas ? kFillMaxCtas : c);
}
// Units [u0, u1) of range c (multiples of 32 units = 128 columns).
__host__ __device__ inline void fill_range(int nunits, int C, int c, int &u0, int &u1) {
    const int n32 = (nunits + 31) / 32;
    u0 = (int)((long)n32 * c / C) * 32;
    const int e = (int)((long)n32 * (c + 1) / C) * 32;
    u1 = e < nunits ? e : nunits;
}
// The four columns of fragment unit u.
__host__ __device__ inline void unit_cols(int u, int kk[4]) {
    const int kb = 16 * (u >> 2) + 2 * (u & 3);
    kk[0] = kb;
    kk[1] = kb + 1;
    kk[2] = kb + 8;
    kk[3] = kb + 9;
}

// 1 / sqrt(mean(x^2) + eps) of an fp32 row in the reference's own order
// (src/kernels/neon.zig:673-702): four lanes, lane j summing x[4i + j]^2
// (multiply, then add) over i in order, combined ((l0 + l1) + l2) + l3, then
// the tail.  Lanes 0..3 of the calling warp each run one lane's chain (a
// serial chain of K / 4 adds: bit-exact with the reference, at the price of
// latency); every lane of the warp gets the result.
__device__ __forceinline__ float ref_order_inv_rms(const float *row, int K, float eps) {
    const int lane = threadIdx.x & 31;
    float l = 0.0f;
    const int n4 = K / 4;
    if (lane < 4) {
#pragma unroll 8
        for (int i = 0; i < n4; ++i) {
            const float v = row[4 * i + lane];
            l = __fadd_rn(l, __fmul_rn(v, v));
        }
    }
    const float l0 = __shfl_sync(0xffffffffu, l, 0), l1 = __shfl_sync(0xffffffffu, l, 1),
                l2 = __shfl_sync(0xffffffffu, l, 2), l3 = __shfl_sync(0xffffffffu, l, 3);
    float ss = __fadd_rn(__fadd_rn(__fadd_rn(l0, l1), l2), l3);
    for (int k = 4 * n4; k < K; ++k) ss = __fadd_rn(ss, __fmul_rn(row[k], row[k]));
    return inv_rms_of(ss, K, eps);
}

// Largest |value| a source produces over columns [k0, k1) (before the RMSNorm
// scale, which is positive and common to the row: max |x[k] * gamma[k]|).
__device__ __forceinline__ float range_absmax(const XSrc &s, int tok, int k0, int k1, int tid, int nthreads) {
    float m = 0.0f;
    if (s.op == kXRmsnorm) {
        const float *row = static_cast<const float *>(s.x) + (size_t)tok * s.ldx;
        for (int k = k0 + tid; k < k1; k += nthreads) m = fmaxf(m, fabsf(__fmul_rn(row[k], s.aux[k])));
    } else {
        for (int k = k0 + tid; k < k1; k += nthreads) m = fmaxf(m, fabsf(xsrc_value(s, tok, k, 1.0f)));
    }
    return m;
}

// Full-row statistics in one block of nthreads (256 or 512): the RMSNorm
// scale in the fill's summation order (1 for other sources) and the row's
// largest |value| (after the RMSNorm scale).  Every range's partials are taken
// in one pass (no barrier between ranges).  red holds
// (kFillMaxCtas + 1) * kFillWarps floats.
__device__ __forceinline__ void block_row_stats(const XSrc &s, int tok, int K, int nunits, int tid, int nthreads,
                                                float *red, int bar_id, float &inv, float &amax) {
    const bool rms = s.op == kXRmsnorm;
    const int C = fill_ctas(nunits);
    const int V = kFillThreads / nthreads;  // threads of the 512 this thread plays
    if (rms) {
        const float *row = static_cast<const float *>(s.x) + (size_t)tok * s.ldx;
        for (int c = 0; c < C; ++c) {
            int u0, u1;
            fill_range(nunits, C, c, u0, u1);
            for (int v = 0; v < V; ++v) {
                const int vt = tid + v * nthreads;
                float a = 0.0f;
                for (int u = u0 + vt; u < u1; u += kFillThreads) {
                    int kk[4];
                    unit_cols(u, kk);
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const float x = kk[q] < K ? row[kk[q]] : 0.0f;
                        a = fmaf(x, x, a);
                    }
                }
#pragma unroll
                for (int off = 16; off > 0; off >>= 1) a += __shfl_xor_sync(0xffffffffu, a, off);
                if ((vt & 31) == 0) red[c * kFillWarps + (vt >> 5)] = a;
            }
        }
    }
    float am = range_absmax(s, tok, 0, K, tid, nthreads);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, off));
    if ((tid & 31) == 0) red[kFillMaxCtas * kFillWarps + (tid >> 5)] = am;
    named_bar_sync(bar_id, nthreads);
    inv = 1.0f;
    if (rms) {
        float tot = 0.0f;
        for (int c = 0; c < C; ++c) {
            float part = 0.0f;
#pragma unroll
            for (int w = 0; w < kFillWarps; ++w) part += red[c * kFillWarps + w];
            tot += part;
        }
        inv = inv_rms_of(tot, K, s.eps);
    }
    float mx = 0.0f;
    for (int w = 0; w < nthreads / 32; ++w) mx = fmaxf(mx, red[kFillMaxCtas * kFillWarps + w]);
    named_bar_sync(bar_id, nthreads);
    amax = rms ? mx * inv : mx;
}

// Power-of-two scaling of an activation row before its fp16 split: e with
// max|x| * 2^e in [2^14, 2^15), so fp16 (largest finite 65504) holds every
// scaled value, including after the 4-bit / 2-bit k-step pre-scales, and the
// hi + lo pair keeps ~22 bits of each value relative to the row's maximum.
// A zero, NaN or infinite maximum leaves the row unscaled; e lies in
// [-113, 126] (a finite maximum gives e >= -113), so 2^e, 2^-e and 2^(e - 6)
// are normal fp32 numbers.  Powers of two are exact: the
// GEMV multiplies its sums by 2^-e in the epilogue.
__host__ __device__ inline int row_scale_exp(float m) {
    if (!(m > 0.0f) || !(m <= 3.402823466e38f)) return 0;
    union {
        float f;
        unsigned u;
    } v;
    v.f = m;
    const int ex = (int)((v.u >> 23) & 0xffu) - 127;  // floor(log2 m); -127 for subnormals
    const int e = 14 - ex;
    return e < -113 ? -113 : (e > 126 ? 126 : e);
}
__host__ __device__ inline float pow2_of(int e) {
    union {
        float f;
        unsigned u;
    } v;
    v.u = (unsigned)(127 + e) << 23;
    return v.f;
}

}  // namespace chpe
