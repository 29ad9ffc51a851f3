// model.cu -- the non-GEMV operations of one decode / verify step
// (src/engine.zig:567-734 step, :753-900 stepBatch4, :902-1095 stepBatch8):
// token embedding, RMSNorm, the reference's stand-in token mixers for the
// full-attention and Gated-DeltaNet blocks, SiLU * mul and the vocabulary
// argmax.  Rows are [M][dim] contiguous.  The residual adds are folded into
// the O / out / down projections (GEMV accumulate into the hidden state).
#include <cfloat>
#include <cstdio>

#include "../../include/chpe_b200.h"
#include "common.cuh"
#include "xsrc.cuh"

namespace chpe {

// src/engine.zig:567-580 embedToken: hidden[i] = int8 row[i] * scale.
__global__ void chpe_embed_i8_kernel(const int8_t *__restrict__ table, float scale, int hidden, int vocab,
                                const int *__restrict__ tokens, float *__restrict__ out, int *__restrict__ err) {
    pdl_begin();
    const int m = blockIdx.y;
    const int tok = tokens[m];
    if (tok < 0 || tok >= vocab) {
        if (threadIdx.x == 0 && blockIdx.x == 0) atomicExch(err, 16);
        return;
    }
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < hidden; i += gridDim.x * blockDim.x)
        out[(size_t)m * hidden + i] = (float)table[(size_t)tok * hidden + i] * scale;
}

// src/kernels/neon.zig:673-702 rmsnorm: y = x * (1/sqrt(mean(x^2) + eps)) * gamma.
// One block per row; the sum of squares in the reference's own lane order
// (ref_order_inv_rms), so the result is the reference's bit for bit.
__global__ void chpe_rmsnorm_kernel(const float *__restrict__ x, const float *__restrict__ gamma, int n, float eps,
                                    float *__restrict__ y) {
    pdl_begin();
    __shared__ float s_inv;
    const float *xr = x + (size_t)blockIdx.x * n;
    float *yr = y + (size_t)blockIdx.x * n;
    if (threadIdx.x < 32) {
        const float v = ref_order_inv_rms(xr, n, eps);
        if (threadIdx.x == 0) s_inv = v;
    }
    __syncthreads();
    const float inv = s_inv;
    for (int i = threadIdx.x; i < n; i += blockDim.x) yr[i] = __fmul_rn(__fmul_rn(xr[i], inv), gamma[i]);
}

// src/engine.zig:619-623: attention stand-in, out[i] = v[i % kv_dim]
// (head_dim = 0); or, head-aligned, each query head h of head_dim columns takes
// kv head h / group (what attention over a single position returns).
__global__ void chpe_mix_attn_kernel(const float *__restrict__ v, int kv_dim, int out_dim, int head_dim, int group,
                                float *__restrict__ out) {
    pdl_begin();
    const int m = blockIdx.y;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < out_dim; i += gridDim.x * blockDim.x) {
        const int src = head_dim ? ((i / head_dim) / group) * head_dim + (i % head_dim) : (i % kv_dim);
        out[(size_t)m * out_dim + i] = v[(size_t)m * kv_dim + src];
    }
}

// src/engine.zig:651-654 (batch 1): out[i] = qkv[i % qkv_dim] * silu(z[i]);
// src/engine.zig:813 / :988 (batch 4 / 8): out[i] = silu(qkv[i]) * z[i].
__global__ void chpe_mix_ssm_kernel(const float *__restrict__ qkv, int qkv_dim, const float *__restrict__ z, int z_dim,
                               int out_dim, int silu_on_qkv, float *__restrict__ out) {
    pdl_begin();
    const int m = blockIdx.y;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < out_dim; i += gridDim.x * blockDim.x) {
        const float q = qkv[(size_t)m * qkv_dim + (i % qkv_dim)];
        const float zz = z[(size_t)m * z_dim + i];
        out[(size_t)m * out_dim + i] = silu_on_qkv ? silu_f(q) * zz : q * silu_f(zz);
    }
}

// src/kernels/neon.zig:705-712 siluMul.
__global__ void chpe_silu_mul_kernel(const float *__restrict__ g, const float *__restrict__ u, size_t n,
                                float *__restrict__ out) {
    pdl_begin();
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        out[i] = silu_f(g[i]) * u[i];
}

// src/engine.zig:1098-1110 computeArgmax: first index of the largest value
// (NaN never wins).  One block per row.
__global__ void chpe_argmax_kernel(const float *__restrict__ logits, int n, int *__restrict__ idx,
                              float *__restrict__ maxv) {
    pdl_begin();
    __shared__ float sv[32];
    __shared__ int si[32];
    const float *r = logits + (size_t)blockIdx.x * n;
    float best = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float v = r[i];
        if (v > best) {  // strided scan: the first hit per thread is its smallest index
            best = v;
            bi = i;
        }
    }
    auto better = [](float v, int i, float bv, int bj) { return v > bv || (v == bv && i < bj); };
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, off);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
        if (better(ov, oi, best, bi)) {
            best = ov;
            bi = oi;
        }
    }
    if ((threadIdx.x & 31) == 0) {
        sv[threadIdx.x >> 5] = best;
        si[threadIdx.x >> 5] = bi;
    }
    __syncthreads();
    if (threadIdx.x < 32) {
        const int nw = blockDim.x >> 5;
        best = threadIdx.x < nw ? sv[threadIdx.x] : -INFINITY;
        bi = threadIdx.x < nw ? si[threadIdx.x] : 0x7fffffff;
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, best, off);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
            if (better(ov, oi, best, bi)) {
                best = ov;
                bi = oi;
            }
        }
        if (threadIdx.x == 0) {
            // all values NaN or -inf: the reference keeps index 0 and max -inf
            idx[blockIdx.x] = bi == 0x7fffffff ? 0 : bi;
            if (maxv) maxv[blockIdx.x] = best;
        }
    }
}

}  // namespace chpe

using namespace chpe;

namespace {
int grid_for(size_t n, int threads) {
    const size_t b = (n + threads - 1) / threads;
    return (int)(b < 1184 ? (b ? b : 1) : 1184);
}
int launched(cudaError_t e) { return e == cudaSuccess ? CHPE_OK : CHPE_ECUDA; }
}  // namespace

// The context is unused by these helpers except for its error word; they take
// it so that every entry point has the same first argument.
int *chpe_ctx_error_word(chpe_ctx *ctx);

extern "C" int chpe_embed_i8_dev(chpe_ctx *ctx, const int8_t *table, float scale, int hidden, int vocab,
                                 const int *tokens, int M, float *out, void *stream) {
    if (!ctx || !table || !tokens || !out || M < 1 || hidden < 1) return CHPE_EINVAL;
    dim3 grid(grid_for(hidden, 256) < 16 ? grid_for(hidden, 256) : 16, M);
    return launched(launch_pdl(chpe_embed_i8_kernel, grid, dim3(256), 0, static_cast<cudaStream_t>(stream), table, scale,
                               hidden, vocab, tokens, out, chpe_ctx_error_word(ctx)));
}

extern "C" int chpe_rmsnorm_dev(chpe_ctx *ctx, const float *x, const float *gamma, int M, int n, float eps, float *y,
                                void *stream) {
    if (!ctx || !x || !gamma || !y || M < 1 || n < 1) return CHPE_EINVAL;
    return launched(launch_pdl(chpe_rmsnorm_kernel, dim3(M), dim3(512), 0, static_cast<cudaStream_t>(stream), x, gamma, n,
                               eps, y));
}

extern "C" int chpe_mix_attn_stub_dev(chpe_ctx *ctx, const float *v, int kv_dim, int M, int out_dim, int head_dim,
                                      int group, float *out, void *stream) {
    if (!ctx || !v || !out || M < 1 || kv_dim < 1) return CHPE_EINVAL;
    if (head_dim && (group < 1 || ((out_dim / head_dim + group - 1) / group) * head_dim > kv_dim)) return CHPE_EINVAL;
    dim3 grid(grid_for(out_dim, 256) < 16 ? grid_for(out_dim, 256) : 16, M);
    return launched(launch_pdl(chpe_mix_attn_kernel, grid, dim3(256), 0, static_cast<cudaStream_t>(stream), v, kv_dim,
                               out_dim, head_dim, group, out));
}

extern "C" int chpe_mix_ssm_stub_dev(chpe_ctx *ctx, const float *qkv, int qkv_dim, const float *z, int z_dim, int M,
                                     int out_dim, int silu_on_qkv, float *out, void *stream) {
    if (!ctx || !qkv || !z || !out || M < 1 || qkv_dim < 1 || out_dim > z_dim) return CHPE_EINVAL;
    dim3 grid(grid_for(out_dim, 256) < 16 ? grid_for(out_dim, 256) : 16, M);
    return launched(launch_pdl(chpe_mix_ssm_kernel, grid, dim3(256), 0, static_cast<cudaStream_t>(stream), qkv, qkv_dim, z,
                               z_dim, out_dim, silu_on_qkv, out));
}

extern "C" int chpe_silu_mul_dev(chpe_ctx *ctx, const float *g, const float *u, size_t n, float *out, void *stream) {
    if (!ctx || !g || !u || !out) return CHPE_EINVAL;
    return launched(launch_pdl(chpe_silu_mul_kernel, dim3(grid_for(n, 256)), dim3(256), 0,
                               static_cast<cudaStream_t>(stream), g, u, n, out));
}

extern "C" int chpe_argmax_dev(chpe_ctx *ctx, const float *logits, int M, int n, int *idx, float *maxv,
                               void *stream) {
    if (!ctx || !logits || !idx || M < 1 || n < 1) return CHPE_EINVAL;
    return launched(launch_pdl(chpe_argmax_kernel, dim3(M), dim3(1024), 0, static_cast<cudaStream_t>(stream), logits, n, idx,
                               maxv));
}
