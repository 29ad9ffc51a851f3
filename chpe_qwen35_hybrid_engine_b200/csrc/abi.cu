// abi.cu -- the C ABI (include/chpe_b200.h): contexts, device tensors, the
// host-pointer operators that mirror the reference's Zig GEMV operators, and
// the device-pointer GEMV entry points.
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <unordered_map>
#include <vector>

#include "../../include/chpe_b200.h"
#include "internal.h"

using namespace chpe;

struct chpe_tensor {
    DevMatrix m;
    uint64_t fingerprint = 0;  // content hash of the host bytes it was made from
};

struct chpe_ctx {
    int device = 0;
    cudaStream_t stream = nullptr;
    std::string err;
    int *d_err = nullptr;
    GemvScratch scr;
    // staging for the host-pointer operators
    void *d_in = nullptr;
    size_t d_in_bytes = 0;
    float *d_out = nullptr;
    size_t d_out_bytes = 0;
    float *d_scales = nullptr;
    float *d_xe = nullptr;  // row unscale factors of the GEMV's fused fill
    void *prefill_xt = nullptr;  // activation tiles of the prefill GEMM
    size_t prefill_xt_bytes = 0;
    std::unordered_map<const void *, chpe_tensor *> registry;
    std::vector<chpe_tensor *> owned;
    void *extra[4] = {nullptr, nullptr, nullptr, nullptr};  // scratch of the step helpers (mixers.cu)
    size_t extra_bytes[4] = {0, 0, 0, 0};
    unsigned extra_gen[4] = {0, 0, 0, 0};   // reallocations of each slot
    unsigned extra_seen[4] = {0, 0, 0, 0};  // the generation whose contents a helper has filled
};

namespace {

int fail(chpe_ctx *ctx, int code, const char *fmt, ...) {
    if (ctx) {
        char buf[512];
        va_list ap;
        va_start(ap, fmt);
        vsnprintf(buf, sizeof buf, fmt, ap);
        va_end(ap);
        ctx->err = buf;
    }
    return code;
}

#define CK(call)                                                                                     \
    do {                                                                                             \
        cudaError_t e_ = (call);                                                                     \
        if (e_ != cudaSuccess)                                                                       \
            return fail(ctx, e_ == cudaErrorMemoryAllocation ? CHPE_ENOMEM : CHPE_ECUDA, "%s: %s (%s:%d)", \
                        #call, cudaGetErrorString(e_), __FILE__, __LINE__);                          \
    } while (0)

bool is_device_ptr(const void *p) {
    if (!p) return false;
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged;
}

int grow(chpe_ctx *ctx, void **p, size_t *cap, size_t need) {
    if (need <= *cap) return CHPE_OK;
    if (*p) cudaFree(*p);
    *p = nullptr;
    *cap = 0;
    size_t sz = need < 4096 ? 4096 : need + need / 4;
    CK(cudaMalloc(p, sz));
    *cap = sz;
    return CHPE_OK;
}

// Copy `bytes` from host or device memory into a fresh device buffer (or
// return the device pointer itself when it already is one).
int to_device(chpe_ctx *ctx, const void *src, size_t bytes, const void **dev, void **owned) {
    *owned = nullptr;
    if (!src || bytes == 0) {
        *dev = nullptr;
        return CHPE_OK;
    }
    if (is_device_ptr(src)) {
        *dev = src;
        return CHPE_OK;
    }
    CK(cudaMalloc(owned, bytes));
    CK(cudaMemcpy(*owned, src, bytes, cudaMemcpyHostToDevice));
    *dev = *owned;
    return CHPE_OK;
}

int log2_exact(int v) {
    int s = 0;
    while ((1 << s) < v) ++s;
    return (1 << s) == v ? s : -1;
}

void free_matrix(DevMatrix &m) {
    cudaFree(m.codes);
    cudaFree(m.bias);
    cudaFree(m.out_cols);
    cudaFree(m.out_w);
    m = DevMatrix();
}

struct UploadSpec {
    int bits, layout, meta_kind, group;
    uint32_t xorv;
    float zc, scale;
    float f32_zc;  // stored-code offset removed from ROW_AFFINE offsets
};

// Build a DevMatrix from device-resident inputs.
int build_matrix(chpe_ctx *ctx, const UploadSpec &u, const uint8_t *d_codes, size_t row_stride, int src_bits,
                 const __half *d_s, const __half *d_z, const float *d_fs, const float *d_fo, const float *d_bias,
                 size_t rows, size_t cols, DevMatrix *out) {
    DevMatrix m;
    m.bits = u.bits;
    m.layout = u.layout;
    m.meta_kind = u.meta_kind;
    m.N = (int)rows;
    m.K = (int)cols;
    m.n_strips = ceil_div((long)rows, kStripRows);
    m.span = block_cols(u.bits);
    m.n_blocks = ceil_div((long)cols, m.span);
    m.group = u.group;
    m.n_groups = (u.layout == kLayoutS8) ? 0 : (int)(cols / u.group);
    if (u.meta_kind == kMetaNone) {
        m.gpb = 0;
        m.gshift = -1;
    } else if (m.n_groups == 1 || u.group > m.span) {
        m.gpb = 1;
        m.gshift = -1;
    } else {
        m.gpb = m.span / u.group;
        m.gshift = log2_exact(u.group);
    }
    m.block_bytes = kBlockCodeBytes + 16 * m.gpb * meta_bytes(u.meta_kind);
    m.scale = u.scale;
    m.zc = u.zc;
    m.xorv = u.xorv;
    m.bytes = (size_t)m.n_strips * m.n_blocks * m.block_bytes;
    cudaError_t e = cudaMalloc(&m.codes, m.bytes);
    if (e != cudaSuccess) return fail(ctx, CHPE_ENOMEM, "cudaMalloc weights (%zu B): %s", m.bytes, cudaGetErrorString(e));
    e = launch_repack_codes(d_codes, row_stride, src_bits, u.xorv, m, ctx->stream);
    if (e == cudaSuccess && u.meta_kind != kMetaNone) e = launch_meta_repack(d_s, d_z, d_fs, d_fo, u.f32_zc, m, ctx->stream);
    if (e != cudaSuccess) {
        free_matrix(m);
        return fail(ctx, CHPE_ECUDA, "repack: %s", cudaGetErrorString(e));
    }
    if (d_bias) {
        e = cudaMalloc(&m.bias, rows * sizeof(float));
        if (e == cudaSuccess) e = cudaMemcpyAsync(m.bias, d_bias, rows * sizeof(float), cudaMemcpyDeviceToDevice, ctx->stream);
        if (e != cudaSuccess) {
            free_matrix(m);
            return fail(ctx, CHPE_ECUDA, "bias: %s", cudaGetErrorString(e));
        }
    }
    e = cudaStreamSynchronize(ctx->stream);
    if (e != cudaSuccess) {
        free_matrix(m);
        return fail(ctx, CHPE_ECUDA, "upload sync: %s", cudaGetErrorString(e));
    }
    *out = m;
    return CHPE_OK;
}

int spec_from_fmt(chpe_ctx *ctx, const chpe_fmt *f, size_t cols, UploadSpec *u) {
    UploadSpec s = {};
    s.bits = f->bits;
    if (s.bits != 2 && s.bits != 4 && s.bits != 8) return fail(ctx, CHPE_EINVAL, "bits must be 2, 4 or 8 (got %d)", s.bits);
    s.group = f->group > 0 ? f->group : (int)cols;
    s.layout = kLayoutF16;
    s.xorv = 0;
    s.zc = 0.0f;
    s.scale = 1.0f;
    s.f32_zc = 0.0f;
    switch (f->scheme) {
    case CHPE_SCHEME_I8_TENSOR:
        if (s.bits != 8) return fail(ctx, CHPE_EINVAL, "I8_TENSOR needs bits = 8");
        s.layout = kLayoutS8;
        s.meta_kind = kMetaNone;
        s.group = (int)cols;
        break;
    case CHPE_SCHEME_I8_GROUP_F16:
        if (s.bits != 8) return fail(ctx, CHPE_EINVAL, "I8_GROUP_F16 needs bits = 8");
        s.meta_kind = kMetaS16;
        s.xorv = 0x80;
        s.zc = 128.0f;
        break;
    case CHPE_SCHEME_U_GROUP_F16_ZERO:
        s.meta_kind = kMetaSZ16;
        break;
    case CHPE_SCHEME_U_GROUP_F16_CONST_ZERO:
        s.meta_kind = kMetaS16;
        s.zc = f->zero;
        break;
    case CHPE_SCHEME_W2_CODEBOOK_GROUP_F16:
        if (s.bits != 2) return fail(ctx, CHPE_EINVAL, "W2_CODEBOOK needs bits = 2");
        s.meta_kind = kMetaS16;
        s.xorv = 2;
        s.zc = 2.0f;
        break;
    case CHPE_SCHEME_ROW_AFFINE_F32:
        s.meta_kind = kMetaF32;
        s.group = (int)cols;
        s.xorv = s.bits == 8 ? 0x80 : s.bits == 2 ? 2 : 0;
        s.f32_zc = s.bits == 8 ? 128.0f : s.bits == 4 ? 8.0f : 2.0f;
        break;
    default:
        return fail(ctx, CHPE_EINVAL, "unknown scheme %d", f->scheme);
    }
    if (s.layout == kLayoutF16) {
        if (cols % (size_t)s.group != 0) return fail(ctx, CHPE_EINVAL, "cols %zu not a multiple of group %d", cols, s.group);
        const int n_groups = (int)(cols / s.group);
        if (n_groups > 1) {
            const int kc = chunk_cols(s.bits);
            const int min_group = s.bits == 2 ? 64 : kc;
            if (log2_exact(s.group) < 0 || s.group < min_group)
                return fail(ctx, CHPE_ENOTSUP, "group %d unsupported for %d-bit codes (power of two >= %d)", s.group,
                            s.bits, min_group);
        }
    }
    *u = s;
    return CHPE_OK;
}

int ensure_scratch(chpe_ctx *ctx, const GemvPlan &P, cudaStream_t st) {
    int rc;
    if ((rc = grow(ctx, &ctx->scr.ws, &ctx->scr.ws_bytes, P.ws_bytes + 64))) return rc;
    const size_t need = (size_t)P.split_counters;
    if (need > ctx->scr.counters_n) {
        if (ctx->scr.counters) cudaFree(ctx->scr.counters);
        ctx->scr.counters = nullptr;
        size_t n = need + 1024;
        CK(cudaMalloc(&ctx->scr.counters, n * sizeof(unsigned)));
        // zeroed on the launch stream so the first kernel sees clean tickets
        CK(cudaMemsetAsync(ctx->scr.counters, 0, n * sizeof(unsigned), st));
        ctx->scr.counters_n = n;
    }
    return CHPE_OK;
}

// Error words that are argument errors found on the device, not expired waits.
constexpr int kErrTokenRange = 16;  // chpe_embed_i8_dev: token id outside the table
constexpr int kErrCacheFull = 41;   // chpe_attn_decode_dev: step past max_seq

// Bytes after the block sums that hold the fill's row unscale factors xe[8].
constexpr size_t kXeBytes = 64;

// Activation fragments of one block of <= 8 rows, ready for the GEMV kernel.
struct Xfrag {
    int layout = kLayoutF16, bits = 8, M = 0, K = 0, Kp = 0, e_cols = 0, x_dtype = 0;
    bool xsplit = false;
    void *xf = nullptr;
    float *xs = nullptr;  // block sums, then the row unscale factors xe[8]
    float *xe = nullptr;
    const float *sx = nullptr;
    const float *xrow = nullptr;  // fp32 rows for outlier columns
};

int check_x(chpe_ctx *ctx, const DevMatrix &w, int x_dtype, const float *x_scales) {
    if (w.layout == kLayoutS8) {
        if (x_dtype != CHPE_X_I8 && x_dtype != CHPE_X_F32)
            return fail(ctx, CHPE_ENOTSUP, "int8 weights take int8 or fp32 activations");
        if (x_dtype == CHPE_X_I8 && !x_scales) return fail(ctx, CHPE_EINVAL, "int8 activations need x_scales");
    } else {
        if (x_dtype == CHPE_X_I8) return fail(ctx, CHPE_ENOTSUP, "int8 activations need an I8_TENSOR weight");
        if (x_dtype != CHPE_X_F32 && x_dtype != CHPE_X_BF16 && x_dtype != CHPE_X_F16)
            return fail(ctx, CHPE_EINVAL, "unknown activation dtype %d", x_dtype);
    }
    return CHPE_OK;
}

int w_kp(const DevMatrix &w) { return w.n_blocks * w.span; }

// Fill fragments (buffers already sized) from M <= 8 rows of x.
int prep_x(chpe_ctx *ctx, Xfrag &f, const void *x, const float *x_scales, float *sx_buf, cudaStream_t st) {
    cudaError_t e;
    if (f.layout == kLayoutS8) {
        if (f.x_dtype == CHPE_X_I8) {
            e = launch_xprep_s8(static_cast<const int8_t *>(x), f.M, f.K, f.Kp, f.xf, st);
            if (e == cudaSuccess && sx_buf) e = cudaMemcpyAsync(sx_buf, x_scales, f.M * sizeof(float), cudaMemcpyDeviceToDevice, st);
            f.sx = sx_buf ? sx_buf : x_scales;
        } else {
            e = launch_act_quant_s8(static_cast<const float *>(x), f.M, f.K, f.Kp, nullptr, sx_buf, f.xf, st);
            f.sx = sx_buf;
        }
    } else {
        e = launch_xprep_f16(x, f.x_dtype, f.M, f.K, f.Kp, f.e_cols, f.xsplit, f.bits, f.xf, f.xs, f.xe, st);
    }
    if (e != cudaSuccess) return fail(ctx, CHPE_ECUDA, "activation prep: %s", cudaGetErrorString(e));
    return CHPE_OK;
}

int check_frag(chpe_ctx *ctx, const DevMatrix &w0, const GemvPlan &P, const Xfrag &f) {
    if (w0.layout != f.layout || w0.K != f.K || w_kp(w0) > f.Kp ||
        (w0.layout == kLayoutF16 && (P.e_cols != f.e_cols || w0.bits != f.bits)))
        return fail(ctx, CHPE_EINVAL,
                    "activation fragments do not match this tensor (K %d/%d, Kp %d/%d, block %d/%d, bits %d/%d)", w0.K,
                    f.K, w_kp(w0), f.Kp, P.e_cols, f.e_cols, w0.bits, f.bits);
    return CHPE_OK;
}

void set_src(GemvSrc &g, const DevMatrix &m, const float *scale_override) {
    g.codes = m.codes;
    g.bias = m.bias;
    g.out_cols = m.out_cols;
    g.out_w = m.out_w;
    g.scale = scale_override ? *scale_override : m.scale;
    g.zc = m.zc;
}

// Kernel parameters of one launch over `n` concatenated plain sources (mode 0)
// or a gate/up pair (mode 1, ms[0] = gate, ms[1] = up), writing ys[r] rows of
// ldys[r] (mode 1: ys[0], ldys[0]).
void fill_params(GemvParams &p, int mode, const DevMatrix *const *ms, int n, const float *const *ovr,
                 float *const *ys, const int *ldys, int accumulate, const GemvPlan &P, const Xfrag &f, void *ws,
                 unsigned *counters, int *err) {
    memset(&p, 0, sizeof p);
    const DevMatrix &w0 = *ms[0];
    for (int i = 0; i < kMaxSrc; ++i) set_src(p.src[i], *ms[i < n ? i : 0], ovr ? ovr[i < n ? i : 0] : nullptr);
    p.nsrc = mode == 1 ? 1 : n;
    int sg = 0;
    for (int r = 0; r <= kMaxSrc; ++r) {
        if (mode == 1 || r >= n) {
            p.sg0[r] = r == 0 ? 0 : (r == p.nsrc ? P.n_sg : 0x7fffffff);
            continue;
        }
        p.sg0[r] = sg;
        p.nstr[r] = ms[r]->n_strips;
        p.rows[r] = ms[r]->N;
        p.ys[r] = ys[r];
        p.ldys[r] = ldys[r];
        sg += ceil_div(ms[r]->n_strips, kSG);
    }
    if (mode == 0) {
        for (int r = n + 1; r <= kMaxSrc; ++r) p.sg0[r] = 0x7fffffff;
        p.sg0[n] = P.n_sg;
    }
    p.N = w0.N;
    p.K = w0.K;
    p.M = f.M;
    p.n_strips = w0.n_strips;
    p.n_blocks = w0.n_blocks;
    p.block_bytes = w0.block_bytes;
    p.gshift = w0.gshift;
    p.meta_kind = w0.meta_kind;
    p.n_sg = P.n_sg;
    p.n_ks = P.n_ks;
    p.bpk = P.bpk;
    p.xf = f.xf;
    p.xs = f.xs;
    p.xe = f.xe;
    p.sx = f.sx;
    p.xrow = f.xrow;
    p.y = ys[0];
    p.ldy = ldys[0];
    p.accumulate = accumulate;
    p.ws = ws;
    p.split_cnt = counters;
    p.work_ctr = counters + P.n_sg;
    p.n_whole = P.n_whole;
    p.bc = P.bc;
    p.cfull = P.cfull;
    p.ctot = P.ctot;
    p.pref = P.pref;
    p.err = err;
}

int gemv_core(chpe_ctx *ctx, const DevMatrix &w0, const DevMatrix *w1, int mode, const Xfrag &f, float *y, int ldy,
              int accumulate, const float *scale_override0, const float *scale_override1, cudaStream_t st,
              const XSrc *src = nullptr, const FillExchange *push = nullptr) {
    GemvPlan P;
    plan_gemv(w0, f.M, mode, f.xsplit, &P, src == nullptr);
    int rc = check_frag(ctx, w0, P, f);
    if (rc) return rc;
    if ((rc = ensure_scratch(ctx, P, st))) return rc;
    if (w0.out_cols && !f.xrow) return fail(ctx, CHPE_EINVAL, "outlier columns need fp32 activations");
    const DevMatrix *ms[2] = {&w0, w1 ? w1 : &w0};
    const float *ovr[2] = {scale_override0, scale_override1};
    GemvParams p;
    fill_params(p, mode, ms, mode == 1 ? 2 : 1, ovr, &y, &ldy, accumulate, P, f, ctx->scr.ws, ctx->scr.counters,
                ctx->d_err);
    if (src) {
        p.xsrc = *src;
        p.fused = 1;
        p.xe = ctx->d_xe;  // written by the kernel's fused fill (for the chunk-sum kernel)
    }
    if (push) p.push = *push;
    cudaError_t e = launch_gemv(w0, w1, P, p, st);
    if (e != cudaSuccess) return fail(ctx, CHPE_ECUDA, "gemv launch: %s", cudaGetErrorString(e));
    return CHPE_OK;
}

// One launch over n <= kMaxSrc plain sources with the same K and format;
// with `src`, every CTA builds its activation fragments from it (fused fill).
int gemv_multi_core(chpe_ctx *ctx, const DevMatrix *const *ms, int n, const Xfrag &f, float *const *ys,
                    cudaStream_t st, const XSrc *src = nullptr, int accumulate = 0) {
    const DevMatrix &w0 = *ms[0];
    int total_sg = 0;
    for (int r = 0; r < n; ++r) {
        const DevMatrix &m = *ms[r];
        if (m.K != w0.K || m.bits != w0.bits || m.layout != w0.layout || m.meta_kind != w0.meta_kind ||
            m.group != w0.group || m.zc != w0.zc || m.n_blocks != w0.n_blocks || m.block_bytes != w0.block_bytes ||
            m.gshift != w0.gshift)
            return fail(ctx, CHPE_EINVAL, "tensor %d: all tensors of one launch need the same K and format", r);
        if (m.out_cols) return fail(ctx, CHPE_EINVAL, "tensor %d has outlier columns (not fused)", r);
        total_sg += ceil_div(m.n_strips, kSG);
    }
    // plan over the concatenation: one matrix of total_sg full strip groups
    DevMatrix cat = w0;
    cat.n_strips = total_sg * kSG;
    cat.N = cat.n_strips * kStripRows;
    GemvPlan P;
    plan_gemv(cat, f.M, 0, f.xsplit, &P, src == nullptr);
    int rc = check_frag(ctx, w0, P, f);
    if (rc) return rc;
    if ((rc = ensure_scratch(ctx, P, st))) return rc;
    int ldys[kMaxSrc];
    for (int r = 0; r < n; ++r) ldys[r] = ms[r]->N;
    GemvParams p;
    fill_params(p, 0, ms, n, nullptr, ys, ldys, accumulate, P, f, ctx->scr.ws, ctx->scr.counters, ctx->d_err);
    if (src) {
        p.xsrc = *src;
        p.fused = 1;
        p.xe = ctx->d_xe;
    }
    cudaError_t e = launch_gemv(w0, nullptr, P, p, st);
    if (e != cudaSuccess) return fail(ctx, CHPE_ECUDA, "gemv launch: %s", cudaGetErrorString(e));
    return CHPE_OK;
}

Xfrag xfrag_shape(const DevMatrix &w, int M, int x_dtype, size_t *xf_bytes, size_t *xs_bytes) {
    Xfrag f;
    f.layout = w.layout;
    f.bits = w.bits;
    f.M = M;
    f.K = w.K;
    f.Kp = w_kp(w);
    f.x_dtype = x_dtype;
    f.xsplit = w.layout == kLayoutF16 && x_dtype == CHPE_X_F32;
    GemvPlan P;
    plan_gemv(w, M, 0, f.xsplit, &P);
    f.e_cols = P.e_cols;
    *xf_bytes = P.xf_bytes;
    *xs_bytes = P.xs_bytes;
    return f;
}

// Core GEMV driver shared by the entry points that take plain activations
// (x is a device pointer [M][K]); blocks of 8 rows use the context scratch.
int run_gemv(chpe_ctx *ctx, const DevMatrix &w0, const DevMatrix *w1, int mode, const void *x, int x_dtype,
             const float *x_scales, int M, float *y, int ldy, int accumulate, const float *scale_override0,
             const float *scale_override1, const float *xrow, cudaStream_t st) {
    if (M < 1) return fail(ctx, CHPE_EINVAL, "M must be >= 1");
    if (!x || !y) return fail(ctx, CHPE_EINVAL, "null x or y");
    int rc = check_x(ctx, w0, x_dtype, x_scales);
    if (rc) return rc;
    const size_t elt = x_dtype == CHPE_X_F32 ? 4 : x_dtype == CHPE_X_I8 ? 1 : 2;
    for (int m0 = 0; m0 < M; m0 += kMaxTokens) {
        const int Mb = (M - m0) < kMaxTokens ? (M - m0) : kMaxTokens;
        size_t xfb, xsb;
        Xfrag f = xfrag_shape(w0, Mb, x_dtype, &xfb, &xsb);
        if ((rc = grow(ctx, &ctx->scr.xf, &ctx->scr.xf_bytes, xfb))) return rc;
        if ((rc = grow(ctx, reinterpret_cast<void **>(&ctx->scr.xs), &ctx->scr.xs_bytes, xsb + kXeBytes))) return rc;
        if ((rc = grow(ctx, reinterpret_cast<void **>(&ctx->scr.sx), &ctx->scr.sx_bytes, 64 * sizeof(float)))) return rc;
        f.xf = ctx->scr.xf;
        f.xs = ctx->scr.xs;
        f.xe = ctx->scr.xs + xsb / sizeof(float);
        f.xrow = xrow ? xrow + (size_t)m0 * w0.K : nullptr;
        const void *xb = static_cast<const uint8_t *>(x) + (size_t)m0 * w0.K * elt;
        if ((rc = prep_x(ctx, f, xb, x_scales ? x_scales + m0 : nullptr,
                         (w0.layout == kLayoutS8 && x_dtype == CHPE_X_F32) ? ctx->scr.sx : nullptr, st)))
            return rc;
        if ((rc = gemv_core(ctx, w0, w1, mode, f, y + (size_t)m0 * ldy, ldy, accumulate, scale_override0,
                            scale_override1, st)))
            return rc;
    }
    return CHPE_OK;
}

int stage_in(chpe_ctx *ctx, const void *src, size_t bytes) {
    int rc = grow(ctx, &ctx->d_in, &ctx->d_in_bytes, bytes);
    if (rc) return rc;
    CK(cudaMemcpyAsync(ctx->d_in, src, bytes, cudaMemcpyHostToDevice, ctx->stream));
    return CHPE_OK;
}

int stage_out(chpe_ctx *ctx, size_t bytes) {
    return grow(ctx, reinterpret_cast<void **>(&ctx->d_out), &ctx->d_out_bytes, bytes);
}

int finish(chpe_ctx *ctx) {
    CK(cudaStreamSynchronize(ctx->stream));
    int h_err = 0;
    CK(cudaMemcpy(&h_err, ctx->d_err, sizeof(int), cudaMemcpyDeviceToHost));
    if (h_err) {
        cudaMemset(ctx->d_err, 0, sizeof(int));
        if (h_err == kErrTokenRange) return fail(ctx, CHPE_EINVAL, "a token id was outside the vocabulary");
        if (h_err == kErrCacheFull) return fail(ctx, CHPE_EINVAL, "a step ran past the KV cache's max_seq positions");
        // a kernel that gave up may have left arrival / work counters set
        if (ctx->scr.counters) cudaMemset(ctx->scr.counters, 0, ctx->scr.counters_n * sizeof(unsigned));
        return fail(ctx, CHPE_ETIMEOUT, "kernel bounded wait expired (code %d)", h_err);
    }
    return CHPE_OK;
}

chpe_tensor *lookup(chpe_ctx *ctx, const void *key) {
    auto it = ctx->registry.find(key);
    return it == ctx->registry.end() ? nullptr : it->second;
}

// FNV-1a over `n` bytes; `sampled` hashes the first and last 4 KiB plus 64
// strided 64-byte windows, enough to notice a host buffer that was freed and
// reused for different weights at the same address.
uint64_t fingerprint(const void *p, size_t n, bool sampled) {
    const uint8_t *b = static_cast<const uint8_t *>(p);
    uint64_t h = 1469598103934665603ull ^ n;
    auto mix = [&](size_t off, size_t len) {
        for (size_t i = 0; i < len && off + i < n; ++i) h = (h ^ b[off + i]) * 1099511628211ull;
    };
    if (!sampled || n <= 16384) {
        mix(0, n);
        return h;
    }
    mix(0, 4096);
    mix(n - 4096, 4096);
    for (int k = 0; k < 64; ++k) mix((n / 64) * k + 4096 % (n / 64), 64);
    return h;
}

}  // namespace

// ---------------------------------------------------------------------------
// context
// ---------------------------------------------------------------------------

extern "C" const char *chpe_version(void) { return "chpe_b200 1.0 sm_100a"; }

namespace {
std::atomic<unsigned long long> g_launches{0};
}
namespace chpe {
void note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }
}  // namespace chpe
extern "C" unsigned long long chpe_kernel_launches(void) { return g_launches.load(std::memory_order_relaxed); }

extern "C" int chpe_init(int device, chpe_ctx **out) {
    if (!out) return CHPE_EINVAL;
    *out = nullptr;
    chpe_ctx *ctx = new chpe_ctx();
    ctx->device = device;
    cudaError_t e = cudaSetDevice(device);
    if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaMalloc(&ctx->d_err, sizeof(int));
    if (e == cudaSuccess) e = cudaMemset(ctx->d_err, 0, sizeof(int));
    if (e == cudaSuccess) e = cudaMalloc(reinterpret_cast<void **>(&ctx->d_scales), 64 * sizeof(float));
    if (e == cudaSuccess) e = cudaMalloc(reinterpret_cast<void **>(&ctx->d_xe), 64 * sizeof(float));
    if (e != cudaSuccess) {
        delete ctx;
        return CHPE_ECUDA;
    }
    *out = ctx;
    return CHPE_OK;
}

extern "C" int chpe_destroy(chpe_ctx *ctx) {
    if (!ctx) return CHPE_EINVAL;
    cudaSetDevice(ctx->device);
    cudaStreamSynchronize(ctx->stream);
    for (chpe_tensor *t : ctx->owned) {
        free_matrix(t->m);
        delete t;
    }
    cudaFree(ctx->scr.xf);
    cudaFree(ctx->scr.xs);
    cudaFree(ctx->scr.sx);
    cudaFree(ctx->scr.ws);
    cudaFree(ctx->scr.counters);
    cudaFree(ctx->d_in);
    cudaFree(ctx->d_out);
    cudaFree(ctx->d_scales);
    cudaFree(ctx->d_xe);
    cudaFree(ctx->d_err);
    cudaFree(ctx->prefill_xt);
    for (void *x : ctx->extra) cudaFree(x);
    cudaStreamDestroy(ctx->stream);
    delete ctx;
    return CHPE_OK;
}

extern "C" const char *chpe_last_error_string(const chpe_ctx *ctx) { return ctx ? ctx->err.c_str() : "null context"; }

extern "C" int chpe_sync(chpe_ctx *ctx) {
    if (!ctx) return CHPE_EINVAL;
    CK(cudaDeviceSynchronize());
    return finish(ctx);
}

// ---------------------------------------------------------------------------
// tensors
// ---------------------------------------------------------------------------

static int upload_common(chpe_ctx *ctx, const chpe_fmt *fmt, const void *codes, size_t row_stride,
                         const void *scales, const void *zeros, const float *bias, size_t rows, size_t cols,
                         int src_bits, chpe_tensor **out) {
    UploadSpec u;
    int rc = spec_from_fmt(ctx, fmt, cols, &u);
    if (rc) return rc;
    if (rows == 0 || cols == 0 || rows > (1u << 30) || cols > (1u << 30)) return fail(ctx, CHPE_EINVAL, "bad shape");
    if (row_stride * 8 < cols * (size_t)src_bits) return fail(ctx, CHPE_EINVAL, "row_stride too small");
    const size_t G = u.layout == kLayoutS8 ? 0 : cols / u.group;
    const void *d_codes, *d_s = nullptr, *d_z = nullptr, *d_bias;
    void *o_codes, *o_s = nullptr, *o_z = nullptr, *o_bias;
    if ((rc = to_device(ctx, codes, rows * row_stride, &d_codes, &o_codes))) return rc;
    const bool f32meta = u.meta_kind == kMetaF32;
    if (u.layout == kLayoutS8) {
        if (!scales) return fail(ctx, CHPE_EINVAL, "I8_TENSOR needs a scale");
        if (is_device_ptr(scales))
            cudaMemcpy(&u.scale, scales, 4, cudaMemcpyDeviceToHost);
        else
            u.scale = *static_cast<const float *>(scales);
    } else {
        if (!scales) return fail(ctx, CHPE_EINVAL, "scales required");
        if ((rc = to_device(ctx, scales, f32meta ? rows * 4 : rows * G * 2, &d_s, &o_s))) return rc;
        if (u.meta_kind == kMetaSZ16 && !zeros) return fail(ctx, CHPE_EINVAL, "zeros required");
        if (zeros && (rc = to_device(ctx, zeros, f32meta ? rows * 4 : rows * G * 2, &d_z, &o_z))) return rc;
    }
    if ((rc = to_device(ctx, bias, bias ? rows * 4 : 0, &d_bias, &o_bias))) return rc;
    chpe_tensor *t = new chpe_tensor();
    rc = build_matrix(ctx, u, static_cast<const uint8_t *>(d_codes), row_stride, src_bits,
                      f32meta ? nullptr : static_cast<const __half *>(d_s),
                      f32meta ? nullptr : static_cast<const __half *>(d_z),
                      f32meta ? static_cast<const float *>(d_s) : nullptr,
                      f32meta ? static_cast<const float *>(d_z) : nullptr, static_cast<const float *>(d_bias), rows,
                      cols, &t->m);
    cudaFree(o_codes);
    cudaFree(o_s);
    cudaFree(o_z);
    cudaFree(o_bias);
    if (rc) {
        delete t;
        return rc;
    }
    ctx->owned.push_back(t);
    *out = t;
    return CHPE_OK;
}

extern "C" int chpe_upload_matrix(chpe_ctx *ctx, const chpe_fmt *fmt, const void *codes, size_t row_stride,
                                  const void *scales, const void *zeros, const float *bias, size_t rows, size_t cols,
                                  chpe_tensor **out) {
    if (!ctx || !fmt || !codes || !out) return fail(ctx, CHPE_EINVAL, "null argument");
    cudaSetDevice(ctx->device);
    return upload_common(ctx, fmt, codes, row_stride, scales, zeros, bias, rows, cols, fmt->bits, out);
}

extern "C" int chpe_quantize_group_dev(chpe_ctx *ctx, const float *w, size_t rows, size_t cols, int bits, int group,
                                       int symmetric, uint8_t *codes, uint16_t *scales, uint16_t *zeros,
                                       void *stream) {
    if (!ctx || !w || !codes || !scales) return fail(ctx, CHPE_EINVAL, "null argument");
    if (group <= 0 || cols % (size_t)group) return fail(ctx, CHPE_EINVAL, "cols must be a multiple of group");
    if (!symmetric && (!zeros || (bits != 2 && bits != 4 && bits != 8)))
        return fail(ctx, CHPE_EINVAL, "asymmetric quantization needs zeros and bits in {2,4,8}");
    cudaError_t e = launch_quant_group(w, (int)rows, (int)cols, group, bits, symmetric, codes,
                                       reinterpret_cast<__half *>(scales), reinterpret_cast<__half *>(zeros),
                                       static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return fail(ctx, CHPE_ECUDA, "quantize: %s", cudaGetErrorString(e));
    return CHPE_OK;
}

// Cell layout constants (src/geometry.zig:243-256, src/weight_archive.zig:92-105,
// src/chpe_engine.zig:146-151).
static constexpr size_t kCellBytes = 17408, kHdr = 64, kCodes = 16384, kPayload = kHdr + kCodes;

static uint8_t cell_bits(const uint8_t *c) { return c[kPayload + 20]; }
static uint64_t cell_flags(const uint8_t *c) {
    uint64_t f;
    memcpy(&f, c + kPayload + 24, 8);
    return f;
}
struct TileDims {
    float scale, bias;
    uint32_t rows, cols;
};
static TileDims cell_dims(const uint8_t *c) {
    TileDims d;
    memcpy(&d, c + kPayload + 32, 16);
    return d;
}

extern "C" int chpe_upload_cells(chpe_ctx *ctx, const void *first_cell, size_t n_cells, size_t tile_stride,
                                 chpe_tensor **out) {
    if (!ctx || !first_cell || !out || n_cells == 0) return fail(ctx, CHPE_EINVAL, "null argument");
    if (tile_stride < kCellBytes) return fail(ctx, CHPE_EINVAL, "tile_stride < 17408");
    cudaSetDevice(ctx->device);
    std::vector<uint8_t> devcopy;
    const uint8_t *base = static_cast<const uint8_t *>(first_cell);
    if (is_device_ptr(first_cell)) {
        devcopy.resize((n_cells - 1) * tile_stride + kCellBytes);
        CK(cudaMemcpy(devcopy.data(), first_cell, devcopy.size(), cudaMemcpyDeviceToHost));
        base = devcopy.data();
    }
    const uint8_t *c0 = base;
    int qb = cell_bits(c0);
    const TileDims d0 = cell_dims(c0);
    const bool g128 = (cell_flags(c0) & 1ull) != 0;
    if (qb == 16 || qb == 32) return fail(ctx, CHPE_ENOTSUP, "fp16/fp32 cells are not quantized (quant_bits %d)", qb);
    if (qb != 4 && qb != 8) qb = 2;  // src/chpe_engine.zig:483-486: unknown widths run as 2-bit
    const size_t cols = d0.cols;
    if (cols == 0 || cols % 4) return fail(ctx, CHPE_EINVAL, "cell cols %zu", cols);
    size_t rows = 0;
    for (size_t i = 0; i < n_cells; ++i) {
        const uint8_t *c = base + i * tile_stride;
        int b = cell_bits(c);
        if (b != 4 && b != 8 && b != 16 && b != 32) b = 2;
        const TileDims d = cell_dims(c);
        if (b != qb || d.cols != cols || ((cell_flags(c) & 1ull) != 0) != g128)
            return fail(ctx, CHPE_ENOTSUP, "cells must share quant_bits, cols and flags");
        if ((size_t)d.rows * cols * qb / 8 > kCodes) return fail(ctx, CHPE_EINVAL, "cell %zu overflows its codes", i);
        rows += d.rows;
    }
    const size_t rs = cols * qb / 8;
    const bool grouped = qb == 2 && g128;
    if (grouped && cols % 128) return fail(ctx, CHPE_ENOTSUP, "group-128 cells need cols %% 128 == 0");
    const size_t G = grouped ? cols / 128 : 1;
    std::vector<uint8_t> codes(rows * rs);
    std::vector<uint16_t> gs(grouped ? rows * G : 0);
    std::vector<float> sc(rows), off(rows), bias(rows);
    std::vector<int> ocols;
    std::vector<uint16_t> ow;
    bool any_out = false;
    size_t r0 = 0;
    for (size_t i = 0; i < n_cells; ++i) {
        const uint8_t *c = base + i * tile_stride;
        const TileDims d = cell_dims(c);
        memcpy(codes.data() + r0 * rs, c + kHdr, d.rows * rs);
        for (uint32_t r = 0; r < d.rows; ++r) {
            sc[r0 + r] = d.scale;
            // per-weight offset for 4/2-bit cells, per-row bias for 8-bit cells
            off[r0 + r] = qb == 8 ? 0.0f : d.bias;
            bias[r0 + r] = qb == 8 ? d.bias : 0.0f;
        }
        if (grouped) {
            for (uint32_t r = 0; r < d.rows; ++r)
                memcpy(&gs[(r0 + r) * G], c + kPayload + 48 + 2 * (r * G), 2 * G);
            if (d.rows == 16) {  // outlier columns (src/chpe_engine.zig:240-252)
                if (!any_out) {
                    ocols.assign(rows * 8, -1);
                    ow.assign(rows * 8, 0);
                    any_out = true;
                }
                uint16_t colsv[8];
                memcpy(colsv, c + kPayload + 816, 16);
                for (uint32_t r = 0; r < 16; ++r)
                    for (int k = 0; k < 8; ++k) {
                        ocols[(r0 + r) * 8 + k] = colsv[k] < cols ? colsv[k] : -1;
                        memcpy(&ow[(r0 + r) * 8 + k], c + kPayload + 560 + 2 * (r * 8 + k), 2);
                    }
            }
        }
        r0 += d.rows;
    }
    chpe_fmt f = {};
    f.bits = qb;
    int rc;
    chpe_tensor *t = nullptr;
    if (grouped) {
        f.scheme = CHPE_SCHEME_W2_CODEBOOK_GROUP_F16;
        f.group = 128;
        rc = upload_common(ctx, &f, codes.data(), rs, gs.data(), nullptr, nullptr, rows, cols, qb, &t);
    } else {
        f.scheme = CHPE_SCHEME_ROW_AFFINE_F32;
        bool any_bias = false;
        for (float b : bias) any_bias |= b != 0.0f;
        rc = upload_common(ctx, &f, codes.data(), rs, sc.data(), off.data(), any_bias ? bias.data() : nullptr, rows,
                           cols, qb, &t);
    }
    if (rc) return rc;
    if (any_out) {
        CK(cudaMalloc(&t->m.out_cols, rows * 8 * sizeof(int)));
        CK(cudaMalloc(&t->m.out_w, rows * 8 * sizeof(uint16_t)));
        CK(cudaMemcpy(t->m.out_cols, ocols.data(), rows * 8 * sizeof(int), cudaMemcpyHostToDevice));
        CK(cudaMemcpy(t->m.out_w, ow.data(), rows * 8 * sizeof(uint16_t), cudaMemcpyHostToDevice));
    }
    *out = t;
    return CHPE_OK;
}

extern "C" int chpe_tensor_free(chpe_ctx *ctx, chpe_tensor *t) {
    if (!ctx || !t) return fail(ctx, CHPE_EINVAL, "null argument");
    for (size_t i = 0; i < ctx->owned.size(); ++i)
        if (ctx->owned[i] == t) {
            for (auto it = ctx->registry.begin(); it != ctx->registry.end();)
                it = (it->second == t) ? ctx->registry.erase(it) : std::next(it);
            cudaStreamSynchronize(ctx->stream);
            free_matrix(t->m);
            delete t;
            ctx->owned.erase(ctx->owned.begin() + i);
            return CHPE_OK;
        }
    return fail(ctx, CHPE_ENOENT, "tensor not owned by this context");
}

extern "C" int chpe_tensor_info(const chpe_tensor *t, size_t *rows, size_t *cols, int *bits, size_t *device_bytes) {
    if (!t) return CHPE_EINVAL;
    if (rows) *rows = t->m.N;
    if (cols) *cols = t->m.K;
    if (bits) *bits = t->m.bits;
    if (device_bytes) *device_bytes = t->m.bytes;
    return CHPE_OK;
}

extern "C" int chpe_tensor_unpack(chpe_ctx *ctx, const chpe_tensor *t, void *codes, void *scales, void *zeros) {
    if (!ctx || !t || !codes) return fail(ctx, CHPE_EINVAL, "null argument");
    const DevMatrix &m = t->m;
    if (zeros && m.meta_kind != kMetaSZ16) return fail(ctx, CHPE_ENOTSUP, "this tensor stores no zero-points");
    cudaSetDevice(ctx->device);
    const size_t row_bytes = ((size_t)m.K * m.bits + 7) / 8;
    const size_t ng = m.meta_kind == kMetaF32 ? 1 : (size_t)m.n_groups;
    const size_t meta_elt = m.meta_kind == kMetaF32 ? 4 : 2;
    const size_t code_bytes = (size_t)m.N * row_bytes, meta_bytes = m.meta_kind == kMetaNone ? 0 : (size_t)m.N * ng * meta_elt;
    uint8_t *d = nullptr;
    CK(cudaMalloc(&d, code_bytes + 2 * meta_bytes + 256));
    uint8_t *ds = d + (code_bytes + 127) / 128 * 128;
    uint8_t *dz = ds + (meta_bytes + 127) / 128 * 128;
    cudaError_t e = launch_unpack(m, m.xorv, row_bytes, d, m.meta_kind == kMetaF32 ? nullptr : reinterpret_cast<__half *>(ds),
                                  m.meta_kind == kMetaSZ16 ? reinterpret_cast<__half *>(dz) : nullptr,
                                  m.meta_kind == kMetaF32 ? reinterpret_cast<float *>(ds) : nullptr, ctx->stream);
    if (e == cudaSuccess) e = cudaMemcpyAsync(codes, d, code_bytes, cudaMemcpyDefault, ctx->stream);
    if (e == cudaSuccess && scales && meta_bytes) e = cudaMemcpyAsync(scales, ds, meta_bytes, cudaMemcpyDefault, ctx->stream);
    if (e == cudaSuccess && zeros) e = cudaMemcpyAsync(zeros, dz, meta_bytes, cudaMemcpyDefault, ctx->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    cudaFree(d);
    if (e != cudaSuccess) return fail(ctx, CHPE_ECUDA, "unpack: %s", cudaGetErrorString(e));
    return CHPE_OK;
}

static void drop_registered(chpe_ctx *ctx, const void *key) {
    chpe_tensor *t = lookup(ctx, key);
    if (!t) return;
    ctx->registry.erase(key);
    chpe_tensor_free(ctx, t);
}

extern "C" int chpe_register_i8(chpe_ctx *ctx, const int8_t *host_weights, size_t rows, size_t cols) {
    if (!ctx || !host_weights) return fail(ctx, CHPE_EINVAL, "null argument");
    const uint64_t fp = is_device_ptr(host_weights) ? 0 : fingerprint(host_weights, rows * cols, true);
    if (chpe_tensor *old = lookup(ctx, host_weights)) {
        if ((size_t)old->m.N == rows && (size_t)old->m.K == cols && old->fingerprint == fp) return CHPE_OK;
        drop_registered(ctx, host_weights);
    }
    cudaSetDevice(ctx->device);
    chpe_fmt f = {8, CHPE_SCHEME_I8_TENSOR, 0, 0.0f};
    const float one = 1.0f;
    chpe_tensor *t;
    int rc = upload_common(ctx, &f, host_weights, cols, &one, nullptr, nullptr, rows, cols, 8, &t);
    if (rc) return rc;
    t->fingerprint = fp;
    ctx->registry[host_weights] = t;
    return CHPE_OK;
}

// ---------------------------------------------------------------------------
// device-pointer GEMV
// ---------------------------------------------------------------------------

extern "C" int chpe_gemv_dev(chpe_ctx *ctx, const chpe_tensor *w, const void *x, int x_dtype, const float *x_scales,
                             int M, float *y, int accumulate, void *stream) {
    if (!ctx || !w) return fail(ctx, CHPE_EINVAL, "null argument");
    return run_gemv(ctx, w->m, nullptr, 0, x, x_dtype, x_scales, M, y, w->m.N, accumulate, nullptr, nullptr,
                    x_dtype == CHPE_X_F32 ? static_cast<const float *>(x) : nullptr, static_cast<cudaStream_t>(stream));
}

extern "C" int chpe_gemv_gateup_swiglu_dev(chpe_ctx *ctx, const chpe_tensor *gate, const chpe_tensor *up,
                                           const void *x, int x_dtype, const float *x_scales, int M, float *mlp_out,
                                           void *stream) {
    if (!ctx || !gate || !up) return fail(ctx, CHPE_EINVAL, "null argument");
    const DevMatrix &g = gate->m, &u = up->m;
    if (g.N != u.N || g.K != u.K || g.bits != u.bits || g.layout != u.layout || g.meta_kind != u.meta_kind ||
        g.group != u.group || g.zc != u.zc)
        return fail(ctx, CHPE_EINVAL, "gate and up must share shape and format");
    if (g.out_cols || u.out_cols) return fail(ctx, CHPE_ENOTSUP, "outlier columns not supported in gate/up");
    return run_gemv(ctx, g, &u, 1, x, x_dtype, x_scales, M, mlp_out, g.N, 0, nullptr, nullptr, nullptr,
                    static_cast<cudaStream_t>(stream));
}

extern "C" int chpe_quantize_act_i8_dev(chpe_ctx *ctx, const float *x, int M, size_t n, int8_t *q, float *scales,
                                        void *stream) {
    if (!ctx || !x || (!q && !scales) || M < 1) return fail(ctx, CHPE_EINVAL, "bad argument");
    cudaError_t e = launch_act_quant_s8(x, M, (int)n, (int)((n + 31) / 32 * 32), q, scales, nullptr,
                                        static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return fail(ctx, CHPE_ECUDA, "act quant: %s", cudaGetErrorString(e));
    return CHPE_OK;
}

// ---------------------------------------------------------------------------
// host-pointer operators mirroring src/engine.zig / src/kernels/neon.zig
// ---------------------------------------------------------------------------

// Registered tensor for a host weight pointer, (re)uploaded when the pointer is
// new or its shape or sampled content changed.
static chpe_tensor *weights_for(chpe_ctx *ctx, const int8_t *w, size_t rows, size_t cols, int *rc) {
    *rc = chpe_register_i8(ctx, w, rows, cols);
    return *rc ? nullptr : lookup(ctx, w);
}

static int batch_common(chpe_ctx *ctx, const int8_t *weights, float scale_w, const int8_t *const *xs,
                        const float *scales_x, int nb, size_t rows, size_t cols, float *const *outs) {
    if (!ctx || !weights || !xs || !outs || !scales_x) return fail(ctx, CHPE_EINVAL, "null argument");
    cudaSetDevice(ctx->device);
    int rc = CHPE_OK;
    chpe_tensor *t = weights_for(ctx, weights, rows, cols, &rc);
    if (!t) return rc;
    if ((rc = grow(ctx, &ctx->d_in, &ctx->d_in_bytes, (size_t)nb * cols))) return rc;
    for (int b = 0; b < nb; ++b)
        CK(cudaMemcpyAsync(static_cast<int8_t *>(ctx->d_in) + (size_t)b * cols, xs[b], cols, cudaMemcpyHostToDevice,
                           ctx->stream));
    CK(cudaMemcpyAsync(ctx->d_scales, scales_x, nb * sizeof(float), cudaMemcpyHostToDevice, ctx->stream));
    if ((rc = stage_out(ctx, (size_t)nb * rows * sizeof(float)))) return rc;
    rc = run_gemv(ctx, t->m, nullptr, 0, ctx->d_in, CHPE_X_I8, ctx->d_scales, nb, ctx->d_out, (int)rows, 0, &scale_w,
                  nullptr, nullptr, ctx->stream);
    if (rc) return rc;
    for (int b = 0; b < nb; ++b)
        CK(cudaMemcpyAsync(outs[b], ctx->d_out + (size_t)b * rows, rows * sizeof(float), cudaMemcpyDeviceToHost,
                           ctx->stream));
    return finish(ctx);
}

extern "C" int chpe_gemv_parallel(chpe_ctx *ctx, const int8_t *weights, float scale_w, const int8_t *x_q8,
                                  float scale_x, size_t rows, size_t cols, float *out) {
    const int8_t *xs[1] = {x_q8};
    float *outs[1] = {out};
    return batch_common(ctx, weights, scale_w, xs, &scale_x, 1, rows, cols, outs);
}

extern "C" int chpe_gemv_batch4_parallel(chpe_ctx *ctx, const int8_t *weights, float scale_w, const int8_t *x0,
                                         const int8_t *x1, const int8_t *x2, const int8_t *x3,
                                         const float scales_x[4], size_t rows, size_t cols, float *out0, float *out1,
                                         float *out2, float *out3) {
    const int8_t *xs[4] = {x0, x1, x2, x3};
    float *outs[4] = {out0, out1, out2, out3};
    return batch_common(ctx, weights, scale_w, xs, scales_x, 4, rows, cols, outs);
}

extern "C" int chpe_gemv_batch8_parallel(chpe_ctx *ctx, const int8_t *weights, float scale_w, const int8_t *const x[8],
                                         const float scales_x[8], size_t rows, size_t cols, float *const out[8]) {
    return batch_common(ctx, weights, scale_w, x, scales_x, 8, rows, cols, out);
}

extern "C" int chpe_gemv_gate_up_swiglu_parallel(chpe_ctx *ctx, const int8_t *gate_weights, float scale_gate,
                                                 const int8_t *up_weights, float scale_up, const int8_t *x_q8,
                                                 float scale_x, size_t rows, size_t cols, float *mlp_out) {
    if (!ctx || !gate_weights || !up_weights || !x_q8 || !mlp_out) return fail(ctx, CHPE_EINVAL, "null argument");
    cudaSetDevice(ctx->device);
    int rc = CHPE_OK;
    chpe_tensor *g = weights_for(ctx, gate_weights, rows, cols, &rc);
    if (!g) return rc;
    chpe_tensor *u = weights_for(ctx, up_weights, rows, cols, &rc);
    if (!u) return rc;
    if ((rc = stage_in(ctx, x_q8, cols))) return rc;
    CK(cudaMemcpyAsync(ctx->d_scales, &scale_x, sizeof(float), cudaMemcpyHostToDevice, ctx->stream));
    if ((rc = stage_out(ctx, rows * sizeof(float)))) return rc;
    rc = run_gemv(ctx, g->m, &u->m, 1, ctx->d_in, CHPE_X_I8, ctx->d_scales, 1, ctx->d_out, (int)rows, 0, &scale_gate,
                  &scale_up, nullptr, ctx->stream);
    if (rc) return rc;
    CK(cudaMemcpyAsync(mlp_out, ctx->d_out, rows * sizeof(float), cudaMemcpyDeviceToHost, ctx->stream));
    return finish(ctx);
}

extern "C" int chpe_quantize_activation_int8(chpe_ctx *ctx, const float *x, size_t n, int8_t *out_q8,
                                             float *scale_out) {
    if (!ctx || !x || !out_q8 || !scale_out || n == 0) return fail(ctx, CHPE_EINVAL, "bad argument");
    cudaSetDevice(ctx->device);
    int rc = stage_in(ctx, x, n * sizeof(float));
    if (rc) return rc;
    if ((rc = stage_out(ctx, n + 64))) return rc;
    int8_t *dq = reinterpret_cast<int8_t *>(ctx->d_out);
    cudaError_t e = launch_act_quant_s8(static_cast<const float *>(ctx->d_in), 1, (int)n, (int)((n + 31) / 32 * 32),
                                        dq, ctx->d_scales, nullptr, ctx->stream);
    if (e != cudaSuccess) return fail(ctx, CHPE_ECUDA, "act quant: %s", cudaGetErrorString(e));
    CK(cudaMemcpyAsync(out_q8, dq, n, cudaMemcpyDeviceToHost, ctx->stream));
    CK(cudaMemcpyAsync(scale_out, ctx->d_scales, sizeof(float), cudaMemcpyDeviceToHost, ctx->stream));
    return finish(ctx);
}

extern "C" int chpe_gemv_tile_polymorphic(chpe_ctx *ctx, const void *cell, const float *x, size_t x_len, float *y,
                                          size_t row_base, int accumulate) {
    if (!ctx || !cell || !x || !y) return fail(ctx, CHPE_EINVAL, "null argument");
    cudaSetDevice(ctx->device);
    const uint64_t fp = fingerprint(cell, kCellBytes, false);
    chpe_tensor *t = lookup(ctx, cell);
    int rc;
    if (t && t->fingerprint != fp) {
        drop_registered(ctx, cell);
        t = nullptr;
    }
    if (!t) {
        if ((rc = chpe_upload_cells(ctx, cell, 1, kCellBytes, &t))) return rc;
        t->fingerprint = fp;
        ctx->registry[cell] = t;
    }
    const DevMatrix &m = t->m;
    if (x_len < (size_t)m.K) return fail(ctx, CHPE_EINVAL, "x_len %zu < cols %d", x_len, m.K);
    if ((rc = stage_in(ctx, x, (size_t)m.K * sizeof(float)))) return rc;
    if ((rc = stage_out(ctx, (size_t)m.N * sizeof(float)))) return rc;
    if (accumulate)
        CK(cudaMemcpyAsync(ctx->d_out, y + row_base, (size_t)m.N * sizeof(float), cudaMemcpyHostToDevice, ctx->stream));
    rc = run_gemv(ctx, m, nullptr, 0, ctx->d_in, CHPE_X_F32, nullptr, 1, ctx->d_out, m.N, accumulate, nullptr, nullptr,
                  static_cast<const float *>(ctx->d_in), ctx->stream);
    if (rc) return rc;
    CK(cudaMemcpyAsync(y + row_base, ctx->d_out, (size_t)m.N * sizeof(float), cudaMemcpyDeviceToHost, ctx->stream));
    return finish(ctx);
}

// ---------------------------------------------------------------------------
// shared activation fragments
// ---------------------------------------------------------------------------

struct chpe_xfrag {
    Xfrag f;
    size_t xf_bytes = 0, xs_bytes = 0;
    float *sx = nullptr;
    float *xrow = nullptr;  // fp32 rows (outlier columns; fused producers into int8 fragments)
    bool outliers = false;  // created like a tensor with outlier columns
};

extern "C" int chpe_xfrag_create(chpe_ctx *ctx, const chpe_tensor *like, int M, int x_dtype, chpe_xfrag **out) {
    if (!ctx || !like || !out) return fail(ctx, CHPE_EINVAL, "null argument");
    if (M < 1 || M > kMaxTokens) return fail(ctx, CHPE_EINVAL, "fragments hold 1..8 rows (got %d)", M);
    int rc = check_x(ctx, like->m, x_dtype, x_dtype == CHPE_X_I8 ? reinterpret_cast<const float *>(1) : nullptr);
    if (rc) return rc;
    cudaSetDevice(ctx->device);
    chpe_xfrag *h = new chpe_xfrag();
    h->f = xfrag_shape(like->m, M, x_dtype, &h->xf_bytes, &h->xs_bytes);
    h->outliers = like->m.out_cols != nullptr;
    cudaError_t e = cudaMalloc(&h->f.xf, h->xf_bytes);
    if (e == cudaSuccess) e = cudaMalloc(reinterpret_cast<void **>(&h->f.xs), h->xs_bytes + kXeBytes);
    if (e == cudaSuccess) h->f.xe = h->f.xs + h->xs_bytes / sizeof(float);
    if (e == cudaSuccess) e = cudaMalloc(reinterpret_cast<void **>(&h->sx), 64 * sizeof(float));
    // fp32 rows are kept beside the fragments only for tensors with outlier
    // columns, and for int8 tensors fed by a fused producer (quantized from them)
    if (e == cudaSuccess && x_dtype == CHPE_X_F32 && (like->m.out_cols || like->m.layout == kLayoutS8))
        e = cudaMalloc(reinterpret_cast<void **>(&h->xrow), (size_t)M * like->m.K * sizeof(float));
    if (e != cudaSuccess) {
        cudaFree(h->f.xf);
        cudaFree(h->f.xs);
        cudaFree(h->sx);
        cudaFree(h->xrow);
        delete h;
        return fail(ctx, CHPE_ENOMEM, "xfrag alloc: %s", cudaGetErrorString(e));
    }
    *out = h;
    return CHPE_OK;
}

extern "C" int chpe_xfrag_fill_dev(chpe_ctx *ctx, chpe_xfrag *xf, const void *x, const float *x_scales,
                                   void *stream) {
    if (!ctx || !xf || !x) return fail(ctx, CHPE_EINVAL, "null argument");
    if (xf->f.x_dtype == CHPE_X_I8 && !x_scales) return fail(ctx, CHPE_EINVAL, "int8 activations need x_scales");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (xf->outliers) {
        cudaError_t e = cudaMemcpyAsync(xf->xrow, x, (size_t)xf->f.M * xf->f.K * sizeof(float), cudaMemcpyDeviceToDevice, st);
        if (e != cudaSuccess) return fail(ctx, CHPE_ECUDA, "xfrag copy: %s", cudaGetErrorString(e));
        xf->f.xrow = xf->xrow;
    }
    return prep_x(ctx, xf->f, x, x_scales, xf->sx, st);
}

extern "C" int chpe_xfrag_fill_op_dev(chpe_ctx *ctx, chpe_xfrag *xf, const chpe_xsrc *src, void *stream) {
    if (!ctx || !xf || !src || !src->x) return fail(ctx, CHPE_EINVAL, "null argument");
    if (src->op < CHPE_XOP_PLAIN || src->op > CHPE_XOP_SSM_STUB) return fail(ctx, CHPE_EINVAL, "unknown op %d", src->op);
    const Xfrag &f = xf->f;
    if (src->op == CHPE_XOP_PLAIN && src->x_dtype != f.x_dtype)
        return fail(ctx, CHPE_EINVAL, "x_dtype %d does not match the fragments (%d)", src->x_dtype, f.x_dtype);
    if (src->op != CHPE_XOP_PLAIN && f.x_dtype != CHPE_X_F32)
        return fail(ctx, CHPE_EINVAL, "fused producers need fragments created for fp32 activations");
    if (src->op != CHPE_XOP_PLAIN && src->op != CHPE_XOP_ATTN_STUB && !src->aux)
        return fail(ctx, CHPE_EINVAL, "op %d needs aux", src->op);
    if (src->op == CHPE_XOP_ATTN_STUB &&
        (src->kv_dim < 1 || (src->head_dim && (src->group < 1 ||
                                               ((f.K / src->head_dim + src->group - 1) / src->group) * src->head_dim >
                                                   src->ldx))))
        return fail(ctx, CHPE_EINVAL, "attention stand-in shape");
    if (src->op == CHPE_XOP_SSM_STUB && src->qkv_dim < 1) return fail(ctx, CHPE_EINVAL, "qkv_dim must be >= 1");
    XSrc s;
    s.op = src->op;
    s.x = src->x;
    s.dt = src->x_dtype;
    s.ldx = src->ldx > 0 ? src->ldx : f.K;
    s.aux = src->aux;
    s.ld_aux = src->ld_aux > 0 ? src->ld_aux : f.K;
    s.eps = src->eps;
    s.kv_dim = src->kv_dim;
    s.head_dim = src->head_dim;
    s.group = src->group;
    s.qkv_dim = src->qkv_dim;
    s.silu_on_qkv = src->silu_on_qkv;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaSuccess;
    if (xf->xrow) {
        // fp32 rows needed (outliers / int8 quantization): produce them once, then fill from them
        e = launch_xmaterialize(s, f.M, f.K, f.Kp, xf->xrow, st);
        if (e != cudaSuccess) return fail(ctx, CHPE_ECUDA, "xfrag producer: %s", cudaGetErrorString(e));
        xf->f.xrow = xf->xrow;
        return prep_x(ctx, xf->f, xf->xrow, nullptr, xf->sx, st);
    }
    if (f.layout != kLayoutF16) return fail(ctx, CHPE_EINVAL, "fused fill of int8 fragments needs fp32 rows");
    e = launch_xfill_f16(s, f.M, f.K, f.Kp, f.e_cols, f.xsplit, f.bits, f.xf, f.xs, f.xe, st);
    if (e != cudaSuccess) return fail(ctx, CHPE_ECUDA, "xfrag fill: %s", cudaGetErrorString(e));
    return CHPE_OK;
}

int comm_fill_exchange(chpe_comm *c, const float *part, float *hidden, size_t n, FillExchange *out);
chpe_ctx *comm_ctx(const chpe_comm *c);

extern "C" int chpe_gemv_xfrag_push_dev(chpe_ctx *ctx, const chpe_tensor *w, const chpe_xfrag *xf, float *y,
                                        chpe_comm *comm, void *stream) {
    if (!ctx || !w || !xf || !y || !comm) return fail(ctx, CHPE_EINVAL, "null argument");
    if (w->m.out_cols) return fail(ctx, CHPE_ENOTSUP, "pushing GEMV: tensors with outlier columns");
    FillExchange ex;
    const int rc = comm_fill_exchange(comm, y, y, (size_t)xf->f.M * w->m.N, &ex);
    if (rc == CHPE_ETIMEOUT) return fail(ctx, rc, "comm object failed: reset it on every rank first");
    if (rc != CHPE_OK) return fail(ctx, rc, "pushing GEMV refused");
    return gemv_core(ctx, w->m, nullptr, 0, xf->f, y, w->m.N, 0, nullptr, nullptr, static_cast<cudaStream_t>(stream),
                     nullptr, &ex);
}

extern "C" int chpe_allreduce_fill_dev(chpe_comm *comm, const float *part, float *hidden, chpe_xfrag *xf,
                                       const float *gamma, float eps, int pushed, void *stream) {
    chpe_ctx *ctx = comm_ctx(comm);
    if (!ctx || !part || !hidden || !xf || !gamma) return fail(ctx, CHPE_EINVAL, "null argument");
    const Xfrag &f = xf->f;
    if (f.layout != kLayoutF16 || f.x_dtype != CHPE_X_F32 || xf->xrow)
        return fail(ctx, CHPE_ENOTSUP, "fused exchange: fp32 fragments of an fp16-operand tensor without outliers");
    FillExchange ex;
    const int rc = comm_fill_exchange(comm, part, hidden, (size_t)f.M * f.K, &ex);
    if (rc == CHPE_ETIMEOUT) return fail(ctx, rc, "comm object failed: reset it on every rank first");
    if (rc != CHPE_OK) return fail(ctx, rc, "fused exchange refused");
    if (!xfill_exchange_fits(f.M, f.Kp))
        return fail(ctx, CHPE_ENOTSUP, "fused exchange: %d rows of %d columns do not fit", f.M, f.K);
    ex.pushed = pushed ? 1 : 0;
    XSrc s;
    s.op = kXRmsnorm;
    s.x = hidden;
    s.dt = CHPE_X_F32;
    s.ldx = f.K;
    s.aux = gamma;
    s.ld_aux = f.K;
    s.eps = eps;
    const cudaError_t e = launch_xfill_f16(s, f.M, f.K, f.Kp, f.e_cols, f.xsplit, f.bits, f.xf, f.xs, f.xe,
                                           static_cast<cudaStream_t>(stream), &ex);
    if (e != cudaSuccess) return fail(ctx, CHPE_ECUDA, "fused exchange fill: %s", cudaGetErrorString(e));
    return CHPE_OK;
}

extern "C" int chpe_gemv_xfrag_dev(chpe_ctx *ctx, const chpe_tensor *w, const chpe_xfrag *xf, float *y,
                                   int accumulate, void *stream) {
    if (!ctx || !w || !xf || !y) return fail(ctx, CHPE_EINVAL, "null argument");
    if (w->m.out_cols && !xf->f.xrow)
        return fail(ctx, CHPE_EINVAL, "tensor has outlier columns: create the fragments like it (fp32)");
    return gemv_core(ctx, w->m, nullptr, 0, xf->f, y, w->m.N, accumulate, nullptr, nullptr,
                     static_cast<cudaStream_t>(stream));
}

// XSrc from the C struct (shared with chpe_xfrag_fill_op_dev), validated.
int make_xsrc(chpe_ctx *ctx, const chpe_xsrc *src, int K, XSrc *out) {
    if (src->op < CHPE_XOP_PLAIN || src->op > CHPE_XOP_SSM_STUB) return fail(ctx, CHPE_EINVAL, "unknown op %d", src->op);
    if (src->op == CHPE_XOP_PLAIN && src->x_dtype != CHPE_X_F32)
        return fail(ctx, CHPE_EINVAL, "fused fills read fp32 activations");
    if (src->op != CHPE_XOP_PLAIN && src->op != CHPE_XOP_ATTN_STUB && !src->aux)
        return fail(ctx, CHPE_EINVAL, "op %d needs aux", src->op);
    if (src->op == CHPE_XOP_ATTN_STUB &&
        (src->kv_dim < 1 ||
         (src->head_dim && (src->group < 1 || ((K / src->head_dim + src->group - 1) / src->group) * src->head_dim >
                                                      (src->ldx > 0 ? src->ldx : K)))))
        return fail(ctx, CHPE_EINVAL, "attention stand-in shape");
    if (src->op == CHPE_XOP_SSM_STUB && src->qkv_dim < 1) return fail(ctx, CHPE_EINVAL, "qkv_dim must be >= 1");
    XSrc s;
    s.op = src->op;
    s.x = src->x;
    s.dt = CHPE_X_F32;
    s.ldx = src->ldx > 0 ? src->ldx : K;
    s.aux = src->aux;
    s.ld_aux = src->ld_aux > 0 ? src->ld_aux : K;
    s.eps = src->eps;
    s.kv_dim = src->kv_dim;
    s.head_dim = src->head_dim;
    s.group = src->group;
    s.qkv_dim = src->qkv_dim;
    s.silu_on_qkv = src->silu_on_qkv;
    *out = s;
    return CHPE_OK;
}

extern "C" int chpe_gemv_src_dev(chpe_ctx *ctx, int mode, int n, const chpe_tensor *const *ws, const chpe_xsrc *src,
                                 int M, float *const *ys, int accumulate, void *stream) {
    if (!ctx || !ws || !src || !src->x || !ys) return fail(ctx, CHPE_EINVAL, "null argument");
    if (M < 1 || M > kMaxTokens) return fail(ctx, CHPE_EINVAL, "fused GEMV takes 1..%d rows (got %d)", kMaxTokens, M);
    if (mode != 0 && mode != 1) return fail(ctx, CHPE_EINVAL, "mode 0 (plain) or 1 (gate/up SwiGLU)");
    if (mode == 1 ? n != 2 : (n < 1 || n > kMaxSrc)) return fail(ctx, CHPE_EINVAL, "tensor count %d for mode %d", n, mode);
    for (int r = 0; r < n; ++r)
        if (!ws[r] || (r < (mode == 1 ? 1 : n) && !ys[r])) return fail(ctx, CHPE_EINVAL, "null tensor or output %d", r);
    const DevMatrix &w0 = ws[0]->m;
    if (w0.layout != kLayoutF16)
        return fail(ctx, CHPE_ENOTSUP, "fused fills feed the fp16 tensor-core path (not int8 x int8 W8A8)");
    for (int r = 0; r < n; ++r)
        if (ws[r]->m.out_cols) return fail(ctx, CHPE_ENOTSUP, "fused fills do not cover outlier columns");
    XSrc s;
    int rc = make_xsrc(ctx, src, w0.K, &s);
    if (rc) return rc;
    cudaSetDevice(ctx->device);
    size_t xfb, xsb;
    Xfrag f = xfrag_shape(w0, M, CHPE_X_F32, &xfb, &xsb);  // shape only: the kernel builds the fragments
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (mode == 1) {
        const DevMatrix &g = ws[0]->m, &u = ws[1]->m;
        if (g.N != u.N || g.K != u.K || g.bits != u.bits || g.layout != u.layout || g.meta_kind != u.meta_kind ||
            g.group != u.group || g.zc != u.zc)
            return fail(ctx, CHPE_EINVAL, "gate and up must share shape and format");
        return gemv_core(ctx, g, &u, 1, f, ys[0], g.N, 0, nullptr, nullptr, st, &s);
    }
    if (n == 1) return gemv_core(ctx, w0, nullptr, 0, f, ys[0], w0.N, accumulate, nullptr, nullptr, st, &s);
    const DevMatrix *ms[kMaxSrc];
    for (int r = 0; r < n; ++r) ms[r] = &ws[r]->m;
    return gemv_multi_core(ctx, ms, n, f, ys, st, &s, accumulate);
}

extern "C" int chpe_gemm_prefill_dev(chpe_ctx *ctx, const chpe_tensor *w, const void *x, int x_dtype, int M, float *y,
                                     int ldy, int accumulate, void *stream) {
    if (!ctx || !w || !x || !y) return fail(ctx, CHPE_EINVAL, "null argument");
    if (M < 1) return fail(ctx, CHPE_EINVAL, "M must be >= 1");
    const DevMatrix &m = w->m;
    if (ldy < m.N) return fail(ctx, CHPE_EINVAL, "ldy %d < rows %d", ldy, m.N);
    if (x_dtype != CHPE_X_F32 && x_dtype != CHPE_X_BF16 && x_dtype != CHPE_X_F16)
        return fail(ctx, CHPE_EINVAL, "prefill activations are fp32, bf16 or fp16");
    if (!prefill_supported(m))
        return fail(ctx, CHPE_ENOTSUP, "prefill GEMM: %d-bit codes with this scale layout (group %d) not supported",
                    m.bits, m.group);
    if (m.out_cols) return fail(ctx, CHPE_ENOTSUP, "prefill GEMM: outlier columns not supported");
    cudaSetDevice(ctx->device);
    int rc = grow(ctx, &ctx->prefill_xt, &ctx->prefill_xt_bytes, prefill_xt_bytes(M, m.K));
    if (rc) return rc;
    cudaError_t e = launch_prefill(m, x, x_dtype, M, ctx->prefill_xt, y, ldy, accumulate, ctx->d_err,
                                   static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) return fail(ctx, CHPE_ECUDA, "prefill launch: %s", cudaGetErrorString(e));
    return CHPE_OK;
}

extern "C" int chpe_gemv_multi_xfrag_dev(chpe_ctx *ctx, int n, const chpe_tensor *const *ws, const chpe_xfrag *xf,
                                         float *const *ys, void *stream) {
    if (!ctx || !ws || !xf || !ys) return fail(ctx, CHPE_EINVAL, "null argument");
    if (n < 1 || n > kMaxSrc) return fail(ctx, CHPE_EINVAL, "1..%d tensors per launch (got %d)", kMaxSrc, n);
    const DevMatrix *ms[kMaxSrc];
    for (int r = 0; r < n; ++r) {
        if (!ws[r] || !ys[r]) return fail(ctx, CHPE_EINVAL, "null tensor or output %d", r);
        ms[r] = &ws[r]->m;
    }
    return gemv_multi_core(ctx, ms, n, xf->f, ys, static_cast<cudaStream_t>(stream));
}

extern "C" int chpe_gemv_gateup_swiglu_xfrag_dev(chpe_ctx *ctx, const chpe_tensor *gate, const chpe_tensor *up,
                                                 const chpe_xfrag *xf, float *mlp_out, void *stream) {
    if (!ctx || !gate || !up || !xf || !mlp_out) return fail(ctx, CHPE_EINVAL, "null argument");
    const DevMatrix &g = gate->m, &u = up->m;
    if (g.N != u.N || g.K != u.K || g.bits != u.bits || g.layout != u.layout || g.meta_kind != u.meta_kind ||
        g.group != u.group || g.zc != u.zc)
        return fail(ctx, CHPE_EINVAL, "gate and up must share shape and format");
    return gemv_core(ctx, g, &u, 1, xf->f, mlp_out, g.N, 0, nullptr, nullptr, static_cast<cudaStream_t>(stream));
}

extern "C" int chpe_xfrag_free(chpe_ctx *ctx, chpe_xfrag *xf) {
    if (!ctx || !xf) return fail(ctx, CHPE_EINVAL, "null argument");
    cudaStreamSynchronize(ctx->stream);
    cudaFree(xf->f.xf);
    cudaFree(xf->f.xs);
    cudaFree(xf->sx);
    cudaFree(xf->xrow);
    delete xf;
    return CHPE_OK;
}

// ---------------------------------------------------------------------------
// allocation-free GEMV
// ---------------------------------------------------------------------------
// Some callers cannot allocate device memory at the moment they run a GEMV:
// host engines that reserve all the device memory they use once at start-up
// (one arena on a GPU shared with other jobs) and treat any later cudaMalloc
// as a failure, and decode loops that cannot take cudaMalloc's implicit
// device synchronisation.  chpe_gemv_dev may grow the context's scratch with
// cudaMalloc on first use of a larger shape; this entry point never does.
// Its scratch -- activation fragments, block sums, chunk sums and the arrival
// and work counters -- lives in one file-scope device array of
// kNoAllocScratchBytes, which every GPU that loads this library holds until
// the process exits.  All calls share the array (it keeps the last call's
// contents), so calls that overlap on the GPU race on it.

constexpr size_t kNoAllocScratchBytes = 16u << 20;  // 16 MiB
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

namespace {

constexpr int kNoAllocMaxDevices = 64;
std::mutex g_noalloc_mu;
void *g_noalloc_ptr[kNoAllocMaxDevices] = {nullptr};
void *g_noalloc_owner[kNoAllocMaxDevices] = {nullptr};  // the device context the address belongs to

// The current CUDA context (driver handle), through the runtime's driver
// entry point; null when unavailable.
void *current_cu_context() {
    using Fn = int (*)(void **);
    static Fn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<Fn>(p);
        else
            cudaGetLastError();
    });
    void *c = nullptr;
    if (fn && fn(&c) != 0) c = nullptr;
    return c;
}

// Device address of the static scratch on the current device (looked up with
// that device current -- in host code the array's name is only a host-side
// stand-in, not a device address -- once per device and device context: a
// context destroyed and re-created, e.g. by cudaDeviceReset, gets a fresh
// lookup instead of a stale address).
int noalloc_scratch(chpe_ctx *ctx, uint8_t **out) {
    if (ctx->device < 0 || ctx->device >= kNoAllocMaxDevices) return fail(ctx, CHPE_EINVAL, "device index");
    void *owner = current_cu_context();
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_ptr[ctx->device] || g_noalloc_owner[ctx->device] != owner) {
        void *ptr = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
        if (e != cudaSuccess || !ptr)
            return fail(ctx, CHPE_ECUDA, "cudaGetSymbolAddress(static scratch): %s", cudaGetErrorString(e));
        g_noalloc_ptr[ctx->device] = ptr;
        g_noalloc_owner[ctx->device] = owner;
    }
    *out = static_cast<uint8_t *>(g_noalloc_ptr[ctx->device]);
    return CHPE_OK;
}

}  // namespace

extern "C" int chpe_gemv_noalloc_dev(chpe_ctx *ctx, const chpe_tensor *w, const void *x, int x_dtype,
                                     const float *x_scales, int M, float *y, void *stream) {
    if (!ctx || !w || !x || !y) return fail(ctx, CHPE_EINVAL, "null argument");
    if (M < 1 || M > kMaxTokens) return fail(ctx, CHPE_EINVAL, "allocation-free GEMV takes 1..8 rows (got %d)", M);
    const DevMatrix &m = w->m;
    int rc = check_x(ctx, m, x_dtype, x_scales);
    if (rc) return rc;
    cudaError_t e = cudaSetDevice(ctx->device);
    if (e != cudaSuccess) return fail(ctx, CHPE_ECUDA, "cudaSetDevice: %s", cudaGetErrorString(e));
    uint8_t *base = nullptr;
    if ((rc = noalloc_scratch(ctx, &base))) return rc;
    cudaStream_t st = static_cast<cudaStream_t>(stream);

    size_t xfb = 0, xsb = 0;
    Xfrag f = xfrag_shape(m, M, x_dtype, &xfb, &xsb);
    GemvPlan P;
    plan_gemv(m, M, 0, f.xsplit, &P);
    // [arrival + work counters | activation fragments | block sums | activation scales | chunk sums]
    auto al = [](size_t v) { return (v + 255) / 256 * 256; };
    const size_t cnt_bytes = al((size_t)P.split_counters * sizeof(unsigned));
    const size_t off_xf = cnt_bytes, off_xs = off_xf + al(xfb), off_sx = off_xs + al(xsb + kXeBytes),
                 off_ws = off_sx + al(kMaxTokens * sizeof(float)), need = off_ws + al(P.ws_bytes);
    if (need > kNoAllocScratchBytes)
        return fail(ctx, CHPE_EINVAL,
                    "shape [%d x %d], M = %d needs %zu bytes of scratch; the allocation-free GEMV has %zu", m.N, m.K, M,
                    need, kNoAllocScratchBytes);
    // arrival and work counters start at zero (they also reset themselves after a clean call)
    e = cudaMemsetAsync(base, 0, cnt_bytes, st);
    if (e != cudaSuccess) return fail(ctx, CHPE_ECUDA, "clear counters: %s", cudaGetErrorString(e));
    f.xf = base + off_xf;
    f.xs = reinterpret_cast<float *>(base + off_xs);
    f.xe = f.xs + xsb / sizeof(float);
    f.xrow = x_dtype == CHPE_X_F32 ? static_cast<const float *>(x) : nullptr;
    float *sx_buf = reinterpret_cast<float *>(base + off_sx);
    if ((rc = prep_x(ctx, f, x, x_scales, (m.layout == kLayoutS8 && x_dtype == CHPE_X_F32) ? sx_buf : nullptr, st)))
        return rc;
    if (m.out_cols && !f.xrow) return fail(ctx, CHPE_EINVAL, "outlier columns need fp32 activations");

    GemvParams p;
    const DevMatrix *ms[1] = {&m};
    int ldy = m.N;
    fill_params(p, 0, ms, 1, nullptr, &y, &ldy, 0, P, f, base + off_ws, reinterpret_cast<unsigned *>(base),
                ctx->d_err);
    e = launch_gemv(m, nullptr, P, p, st);
    if (e != cudaSuccess) return fail(ctx, CHPE_ECUDA, "gemv launch: %s", cudaGetErrorString(e));
    return CHPE_OK;
}

// Error word of a context (used by the step helpers in model.cu).
int *chpe_ctx_error_word(chpe_ctx *ctx) { return ctx->d_err; }

// Scratch slot `slot` (0..3) of a context, at least `bytes` long and zeroed
// when (re)allocated -- the device is synchronised around a reallocation, so
// a helper's first call at a size must come before any stream capture.
int chpe_ctx_scratch(chpe_ctx *ctx, int slot, size_t bytes, void **out) {
    if (slot < 0 || slot >= 4) return CHPE_EINVAL;
    if (bytes > ctx->extra_bytes[slot]) {
        cudaSetDevice(ctx->device);
        if (ctx->extra[slot]) cudaFree(ctx->extra[slot]);
        ctx->extra[slot] = nullptr;
        ctx->extra_bytes[slot] = 0;
        CK(cudaMalloc(&ctx->extra[slot], bytes));
        CK(cudaMemset(ctx->extra[slot], 0, bytes));
        CK(cudaDeviceSynchronize());
        ctx->extra_bytes[slot] = bytes;
        ++ctx->extra_gen[slot];
    }
    *out = ctx->extra[slot];
    return CHPE_OK;
}
unsigned chpe_ctx_scratch_generation(chpe_ctx *ctx, int slot) { return ctx->extra_gen[slot]; }
unsigned chpe_ctx_scratch_seen(chpe_ctx *ctx, int slot) { return ctx->extra_seen[slot]; }
void chpe_ctx_scratch_mark_seen(chpe_ctx *ctx, int slot) { ctx->extra_seen[slot] = ctx->extra_gen[slot]; }
