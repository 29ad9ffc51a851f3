// internal.h -- host-side declarations shared between the C ABI (abi.cu) and
// the kernel launchers (gemv.cu, prep.cu).
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "layout.h"

namespace chpe {

// One weight matrix in strip layout on the device.
struct DevMatrix {
    int bits = 0;
    int layout = kLayoutF16;
    int meta_kind = kMetaNone;
    int N = 0, K = 0;
    int n_strips = 0, n_chunks = 0;
    int group = 0;     // columns per group (K when one group per row)
    int n_groups = 0;  // groups per row
    int group_shift = 0;
    float scale = 1.0f;  // per-tensor scale (S8 layout)
    float zc = 0.0f;     // constant zero-point (kMetaS16)
    uint8_t *codes = nullptr;
    void *meta = nullptr;
    float *bias = nullptr;
    int *out_cols = nullptr;        // [N][8] outlier columns, -1 = none
    __half *out_w = nullptr;        // [N][8] outlier weights
    size_t code_bytes = 0, meta_bytes_total = 0;
};

struct GemvSrc {
    const uint8_t *codes;
    const void *meta;
    const float *bias;
    const int *out_cols;
    const __half *out_w;
    float scale;
    float zc;
};

struct GemvParams {
    GemvSrc src[2];
    int N, K, M;
    int n_strips, n_chunks, n_groups, group_shift;
    int meta_kind;
    int n_sg, n_ks, cpk;
    int gps;  // metadata groups reserved per strip in shared memory
    const void *xf;
    const void *xlo;
    const float *xs;
    const float *sx;
    const float *xrow;  // fp32 activations [M][K] (outlier columns), or null
    float *y;
    int ldy;
    int accumulate;
    void *ws;
    unsigned *counters;
    int *err;
};

// Scratch a GEMV call needs, owned by the caller (context).
struct GemvScratch {
    void *xf = nullptr, *xlo = nullptr;
    float *xs = nullptr, *sx = nullptr;
    void *ws = nullptr;
    unsigned *counters = nullptr;
    size_t xf_bytes = 0, xlo_bytes = 0, xs_bytes = 0, sx_bytes = 0, ws_bytes = 0, counters_n = 0;
};

// Launch plan of one GEMV (computed on the host).
struct GemvPlan {
    int mode = 0;  // 0 plain, 1 gate/up SwiGLU
    int sg = 2;
    int n_sg = 0, n_ks = 0, cpk = 0, gps = 0;
    int e_cols = 0;  // epilogue block (columns)
    bool xsplit = false;
    size_t smem = 0;
    size_t xf_bytes = 0, xlo_bytes = 0, xs_bytes = 0, ws_bytes = 0;
    int counters = 0;
};

int plan_gemv(const DevMatrix &w, int M, int mode, bool xsplit, GemvPlan *plan);

// x-fragment preparation (fp activations -> fp16 fragments + block sums).
cudaError_t launch_xprep_f16(const void *x, int x_dtype, int M, int K, int Kp, int e_cols, bool xsplit, void *xf,
                             void *xlo, float *xs, cudaStream_t st);
// int8 activations -> int8 fragments.
cudaError_t launch_xprep_s8(const int8_t *xq, int M, int K, int Kp, void *xf, cudaStream_t st);
// fp32 activations -> per-row dynamic int8 quantization (+ fragments).
cudaError_t launch_act_quant_s8(const float *x, int M, int K, int Kp, int8_t *q, float *scales, void *xf,
                                cudaStream_t st);

cudaError_t launch_gemv(const DevMatrix &w0, const DevMatrix *w1, const GemvPlan &plan, const GemvParams &p,
                        cudaStream_t st);

// Repack row-major codes of `src_bits` bits each (LSB first inside a byte;
// src_bits = 8 for one byte per code) into the strip layout of `bits`-wide
// codes, XOR-ing each code with `xorv` (F16 layout only).
cudaError_t launch_repack2(const uint8_t *src, size_t row_stride, int N, int K, int src_bits, int bits, int layout,
                           uint32_t xorv, uint8_t *dst, int n_strips, int n_chunks, cudaStream_t st);
// Grouped quantization of fp32 weights [N][K] (one code byte per weight).
cudaError_t launch_quant_group(const float *w, int N, int K, int group, int bits, int symmetric, uint8_t *codes,
                               __half *scales, __half *zeros, cudaStream_t st);
// fp16 scale/zero [N][G] -> strip metadata.
cudaError_t launch_meta_repack(int kind, const __half *s, const __half *z, const float *fs, const float *fo,
                               float zc_for_f32, int N, int G, void *dst, int n_strips, cudaStream_t st);

}  // namespace chpe
