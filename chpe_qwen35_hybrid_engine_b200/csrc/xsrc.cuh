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

}  // namespace chpe
