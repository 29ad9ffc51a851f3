/*
 * chpe_oracle.c -- CPU restatement of the CHPE quantized dequant-matmul path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the oracle the CUDA path is checked
 * against.  Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg
 * may load it; the product library never links or calls it.
 *
 * Every function restates one reference function (Zig / numpy) and cites the
 * file:line it follows.  Floating-point operations are written in the same
 * order as the reference (build with -ffp-contract=off so no FMA is formed),
 * integer sums are exact.  Parity is pinned by tests/golden (fixtures produced
 * by importing the reference packer) and by the reference's own known-answer
 * tests (src/kernels/neon.zig:714-841, src/chpe_engine.zig:811-888).
 *
 * The grouped formats (int8 group-32 with fp16 scales; 4/2-bit group-64 with
 * fp16 scale + fp16 zero) have no reference implementation: here the
 * restatement IS the specification, and a degenerate-parameter test ties each
 * one back to a reference path.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

typedef _Float16 f16;

/* exp of the reference's silu (`@exp` in src/kernels/neon.zig:705-712), taken
 * in double and rounded to float: the correctly rounded float exp except in
 * about one case in 10^9.  The CUDA path does the same, so the two agree bit
 * for bit (any two float exps may differ in the last bit, which the int8
 * activation re-quantization of the W8A8 path can turn into a flipped code). */
static inline float exp_rn(float x) { return (float)exp((double)x); }

/* ------------------------------------------------------------------------ */
/* int8 dot kernels: src/kernels/neon.zig (x86 `else` branches)              */
/* ------------------------------------------------------------------------ */

/* src/kernels/neon.zig:54-124  dotProductInt8Neon */
float oracle_dot_i8(const int8_t *a, const int8_t *b, size_t n, float scale_w, float scale_x) {
    int32_t acc = 0;
    for (size_t i = 0; i < n; ++i) acc += (int32_t)a[i] * (int32_t)b[i];
    return (float)acc * (scale_w * scale_x);
}

/* src/kernels/neon.zig:129-255  dotProductInt8QuadRowNeon */
void oracle_dot_i8_quadrow(const int8_t *w0, const int8_t *w1, const int8_t *w2, const int8_t *w3,
                           const int8_t *x, size_t n, float scale_w, float scale_x, float *out4) {
    int32_t a0 = 0, a1 = 0, a2 = 0, a3 = 0;
    for (size_t i = 0; i < n; ++i) {
        int32_t xi = x[i];
        a0 += (int32_t)w0[i] * xi;
        a1 += (int32_t)w1[i] * xi;
        a2 += (int32_t)w2[i] * xi;
        a3 += (int32_t)w3[i] * xi;
    }
    float norm = scale_w * scale_x;
    out4[0] = (float)a0 * norm;
    out4[1] = (float)a1 * norm;
    out4[2] = (float)a2 * norm;
    out4[3] = (float)a3 * norm;
}

/* src/kernels/neon.zig:261-350  dotProductInt8GateUpSwiGLUNeon */
float oracle_dot_i8_gateup_swiglu(const int8_t *wg, const int8_t *wu, const int8_t *x, size_t n,
                                  float scale_gate, float scale_up, float scale_x) {
    int32_t ag = 0, au = 0;
    for (size_t i = 0; i < n; ++i) {
        ag += (int32_t)wg[i] * (int32_t)x[i];
        au += (int32_t)wu[i] * (int32_t)x[i];
    }
    float g = (float)ag * (scale_gate * scale_x);
    float u = (float)au * (scale_up * scale_x);
    float silu_g = g / (1.0f + exp_rn(-g));
    return silu_g * u;
}

/* src/kernels/neon.zig:355-477 (Batch4) and :482-641 (Batch8): one weight row
 * against nb int8 vectors, per-vector activation scales. */
void oracle_dot_i8_batch(const int8_t *w, const int8_t *const *xs, int nb, size_t n,
                         float scale_w, const float *scales_x, float *out) {
    for (int b = 0; b < nb; ++b) {
        int32_t acc = 0;
        for (size_t i = 0; i < n; ++i) acc += (int32_t)w[i] * (int32_t)xs[b][i];
        out[b] = (float)acc * (scale_w * scales_x[b]);
    }
}

/* src/kernels/neon.zig:644-670  quantizeActivationInt8.  Zig @round rounds half
 * away from zero, which is C roundf. */
float oracle_quantize_act_i8(const float *x, size_t n, int8_t *q) {
    float max_val = 0.0f;
    for (size_t i = 0; i < n; ++i) {
        float av = fabsf(x[i]);
        if (av > max_val) max_val = av;
    }
    float scale = (max_val > 1e-9f) ? max_val / 127.0f : 1.0f;
    float inv_scale = 1.0f / scale;
    for (size_t i = 0; i < n; ++i) {
        float r = roundf(x[i] * inv_scale);
        float c = fmaxf(-128.0f, fminf(127.0f, r));
        q[i] = (int8_t)c;
    }
    return scale;
}

/* src/kernels/neon.zig:673-702  rmsnorm (Vec4 partial sums, ordered reduce) */
void oracle_rmsnorm(const float *x, const float *gamma, float *y, size_t n, float eps) {
    float lane[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    size_t i = 0;
    for (; i + 4 <= n; i += 4)
        for (int j = 0; j < 4; ++j) lane[j] += x[i + j] * x[i + j];
    float sum_sq = ((lane[0] + lane[1]) + lane[2]) + lane[3];
    for (; i < n; ++i) sum_sq += x[i] * x[i];
    float mean_sq = sum_sq / (float)n;
    float inv_rms = 1.0f / sqrtf(mean_sq + eps);
    for (i = 0; i < n; ++i) y[i] = x[i] * inv_rms * gamma[i];
}

/* src/kernels/neon.zig:705-712  siluMul */
void oracle_silu_mul(const float *g, const float *u, float *out, size_t n) {
    for (size_t i = 0; i < n; ++i) {
        float s = g[i] / (1.0f + exp_rn(-g[i]));
        out[i] = s * u[i];
    }
}

/* ------------------------------------------------------------------------ */
/* Row-partitioned GEMV operators: src/engine.zig:176-460                    */
/* The worker pool (src/engine.zig:90-174) splits rows into NUM_WORKERS      */
/* contiguous slices, the last worker taking the remainder; each slice runs  */
/* the quad-row kernel on groups of 4 rows and the single-row kernel on the  */
/* tail.  Results do not depend on the split (integer sums are exact); the   */
/* threads exist for the CPU baseline timing.                                */
/* ------------------------------------------------------------------------ */

typedef struct {
    int kind; /* 0 gemv, 1 gate/up swiglu, 2 batch */
    int worker_id, num_workers;
    const int8_t *w, *w2;
    float sw, sw2;
    const int8_t *x;
    const int8_t *const *xs;
    int nb;
    float sx;
    const float *sxs;
    size_t rows, cols;
    float *out;
    float *const *outs;
} gemv_job;

static void gemv_slice(const gemv_job *j) {
    size_t per = j->rows / (size_t)j->num_workers;
    size_t start = (size_t)j->worker_id * per;
    size_t end = (j->worker_id == j->num_workers - 1) ? j->rows : start + per;
    size_t c = j->cols;
    if (j->kind == 0) { /* src/engine.zig:188-225 gemvWorkerFn */
        size_t r = start;
        for (; r + 4 <= end; r += 4) {
            float o[4];
            oracle_dot_i8_quadrow(j->w + (r + 0) * c, j->w + (r + 1) * c, j->w + (r + 2) * c,
                                  j->w + (r + 3) * c, j->x, c, j->sw, j->sx, o);
            j->out[r + 0] = o[0];
            j->out[r + 1] = o[1];
            j->out[r + 2] = o[2];
            j->out[r + 3] = o[3];
        }
        for (; r < end; ++r) j->out[r] = oracle_dot_i8(j->w + r * c, j->x, c, j->sw, j->sx);
    } else if (j->kind == 1) { /* src/engine.zig:265-283 gemvGateUpWorkerFn */
        for (size_t r = start; r < end; ++r)
            j->out[r] = oracle_dot_i8_gateup_swiglu(j->w + r * c, j->w2 + r * c, j->x, c, j->sw, j->sw2, j->sx);
    } else { /* src/engine.zig:331-355 / :405-432 batch worker fns */
        float o[8];
        for (size_t r = start; r < end; ++r) {
            oracle_dot_i8_batch(j->w + r * c, j->xs, j->nb, c, j->sw, j->sxs, o);
            for (int b = 0; b < j->nb; ++b) j->outs[b][r] = o[b];
        }
    }
}

static void *gemv_thread(void *p) {
    gemv_slice((const gemv_job *)p);
    return NULL;
}

static void run_pool(gemv_job *proto, int num_workers) {
    if (num_workers < 1) num_workers = 1;
    if (num_workers > 256) num_workers = 256;
    gemv_job jobs[256];
    pthread_t th[256];
    for (int w = 0; w < num_workers; ++w) {
        jobs[w] = *proto;
        jobs[w].worker_id = w;
        jobs[w].num_workers = num_workers;
    }
    for (int w = 1; w < num_workers; ++w) pthread_create(&th[w], NULL, gemv_thread, &jobs[w]);
    gemv_slice(&jobs[0]); /* worker 0 runs on the caller, src/engine.zig:124-125 */
    for (int w = 1; w < num_workers; ++w) pthread_join(th[w], NULL);
}

/* src/engine.zig:227-251  gemvParallel */
void oracle_gemv_parallel(const int8_t *weights, float scale_w, const int8_t *x_q8, float scale_x,
                          size_t rows, size_t cols, float *out, int num_workers) {
    gemv_job j = {0};
    j.kind = 0; j.w = weights; j.sw = scale_w; j.x = x_q8; j.sx = scale_x;
    j.rows = rows; j.cols = cols; j.out = out;
    run_pool(&j, num_workers);
}

/* src/engine.zig:285-313  gemvGateUpSwiGLUParallel */
void oracle_gemv_gateup_swiglu_parallel(const int8_t *gate, float scale_gate, const int8_t *up, float scale_up,
                                        const int8_t *x_q8, float scale_x, size_t rows, size_t cols,
                                        float *mlp_out, int num_workers) {
    gemv_job j = {0};
    j.kind = 1; j.w = gate; j.w2 = up; j.sw = scale_gate; j.sw2 = scale_up; j.x = x_q8; j.sx = scale_x;
    j.rows = rows; j.cols = cols; j.out = mlp_out;
    run_pool(&j, num_workers);
}

/* src/engine.zig:357-391 gemvBatch4Parallel and :434-460 gemvBatch8Parallel */
void oracle_gemv_batch_parallel(const int8_t *weights, float scale_w, const int8_t *const *xs, const float *scales_x,
                                int nb, size_t rows, size_t cols, float *const *outs, int num_workers) {
    gemv_job j = {0};
    j.kind = 2; j.w = weights; j.sw = scale_w; j.xs = xs; j.nb = nb; j.sxs = scales_x;
    j.rows = rows; j.cols = cols; j.outs = outs;
    run_pool(&j, num_workers);
}

/* ------------------------------------------------------------------------ */
/* Packed-tile GEMVs over one Cell: src/chpe_engine.zig:214-488              */
/* Cell layout (src/geometry.zig:243-256): 64 B header, 16384 B codes,       */
/* 960 B payload; TileMetadata at payload[0..32]                             */
/* (src/weight_archive.zig:92-105), TileDims {scale,bias,rows,cols} at       */
/* payload[32..48] (src/chpe_engine.zig:146-151).                            */
/* ------------------------------------------------------------------------ */

#define CELL_HDR 64
#define CELL_CODES 16384
#define CELL_PAYLOAD_OFF (CELL_HDR + CELL_CODES)
#define FLAG_GROUP128_OUTLIERS 0x01ull

typedef struct { float scale, bias; uint32_t rows, cols; } tile_dims;

static tile_dims cell_dims(const uint8_t *cell) {
    tile_dims d;
    memcpy(&d, cell + CELL_PAYLOAD_OFF + 32, sizeof d);
    return d;
}
static uint8_t cell_quant_bits(const uint8_t *cell) { return cell[CELL_PAYLOAD_OFF + 20]; }
static uint64_t cell_flags(const uint8_t *cell) {
    uint64_t f;
    memcpy(&f, cell + CELL_PAYLOAD_OFF + 24, 8);
    return f;
}

static const float CODEBOOK_W2[4] = {0.0f, 1.0f, -2.0f, -1.0f}; /* src/chpe_engine.zig:216 */

static void put_y(float *y, size_t idx, float v, int accumulate) {
    if (accumulate) y[idx] += v;
    else y[idx] = v;
}

/* src/chpe_engine.zig:219-316  gemvTileW2 */
void oracle_gemv_tile_w2(const uint8_t *cell, const float *x, size_t x_len, float *y, size_t row_base, int accumulate) {
    const uint8_t *payload = cell + CELL_PAYLOAD_OFF;
    tile_dims d = cell_dims(cell);
    const uint8_t *coded = cell + CELL_HDR;
    size_t rows = d.rows, cols = d.cols;
    int has_group128 = (cell_flags(cell) & FLAG_GROUP128_OUTLIERS) != 0;
    int has_outliers = has_group128 && rows == 16;
    float x_out[8] = {0};
    if (has_outliers) {
        for (int k = 0; k < 8; ++k) {
            uint16_t col;
            memcpy(&col, payload + 816 + 2 * k, 2);
            if (col < x_len) x_out[k] = x[col];
        }
    }
    size_t n_groups = cols / 128;
    for (size_t r = 0; r < rows; ++r) {
        float row_sum = 0.0f;
        size_t rb = r * (cols / 4);
        if (has_group128) {
            for (size_t g = 0; g < n_groups; ++g) {
                f16 s16;
                memcpy(&s16, payload + 48 + 2 * (r * n_groups + g), 2);
                float scale = (float)s16;
                const uint8_t *gb = coded + rb + g * 32;
                const float *xs = x + g * 128;
                float dv[8] = {0};
                for (size_t j = 0; j < 32; j += 2) {
                    uint8_t b0 = gb[j], b1 = gb[j + 1];
                    float q[8] = {CODEBOOK_W2[b0 & 3], CODEBOOK_W2[(b0 >> 2) & 3], CODEBOOK_W2[(b0 >> 4) & 3],
                                  CODEBOOK_W2[(b0 >> 6) & 3], CODEBOOK_W2[b1 & 3], CODEBOOK_W2[(b1 >> 2) & 3],
                                  CODEBOOK_W2[(b1 >> 4) & 3], CODEBOOK_W2[(b1 >> 6) & 3]};
                    for (int l = 0; l < 8; ++l) dv[l] += q[l] * xs[4 * j + l];
                }
                float red = dv[0];
                for (int l = 1; l < 8; ++l) red += dv[l];
                row_sum += red * scale;
            }
        } else {
            float scale = d.scale, bias = d.bias;
            for (size_t b = 0; b < cols / 4; ++b) {
                uint8_t bv = coded[rb + b];
                float w0 = CODEBOOK_W2[bv & 3] * scale + bias;
                float w1 = CODEBOOK_W2[(bv >> 2) & 3] * scale + bias;
                float w2 = CODEBOOK_W2[(bv >> 4) & 3] * scale + bias;
                float w3 = CODEBOOK_W2[(bv >> 6) & 3] * scale + bias;
                size_t base = b * 4;
                row_sum += w0 * x[base] + w1 * x[base + 1] + w2 * x[base + 2] + w3 * x[base + 3];
            }
        }
        if (has_outliers) {
            float red = 0.0f;
            for (int k = 0; k < 8; ++k) {
                f16 w16;
                memcpy(&w16, payload + 560 + 2 * (r * 8 + k), 2);
                red += (float)w16 * x_out[k];
            }
            row_sum += red;
        }
        put_y(y, row_base + r, row_sum, accumulate);
    }
}

/* src/chpe_engine.zig:319-354  gemvTileW4 (offset-8 nibbles, low nibble first,
 * per-tile scale and bias; the group scales in the payload are not read) */
void oracle_gemv_tile_w4(const uint8_t *cell, const float *x, float *y, size_t row_base, int accumulate) {
    tile_dims d = cell_dims(cell);
    const uint8_t *coded = cell + CELL_HDR;
    size_t rows = d.rows, cols = d.cols;
    for (size_t r = 0; r < rows; ++r) {
        float row_sum = 0.0f;
        const uint8_t *rb = coded + r * (cols / 2);
        for (size_t b = 0; b < cols / 2; ++b) {
            uint8_t bv = rb[b];
            int n0 = (int)(bv & 0x0F) - 8, n1 = (int)((bv >> 4) & 0x0F) - 8;
            float w0 = (float)n0 * d.scale + d.bias;
            float w1 = (float)n1 * d.scale + d.bias;
            row_sum += w0 * x[2 * b] + w1 * x[2 * b + 1];
        }
        put_y(y, row_base + r, row_sum, accumulate);
    }
}

/* src/chpe_engine.zig:357-406  gemvTileW8 (fp32 x, Vec8 partial sums,
 * y = row_sum*scale + bias) */
void oracle_gemv_tile_w8(const uint8_t *cell, const float *x, float *y, size_t row_base, int accumulate) {
    tile_dims d = cell_dims(cell);
    const int8_t *coded = (const int8_t *)(cell + CELL_HDR);
    size_t rows = d.rows, cols = d.cols;
    for (size_t r = 0; r < rows; ++r) {
        const int8_t *rw = coded + r * cols;
        float acc[8] = {0};
        size_t i = 0;
        for (; i + 8 <= cols; i += 8)
            for (int l = 0; l < 8; ++l) acc[l] += (float)rw[i + l] * x[i + l];
        float row_sum = acc[0];
        for (int l = 1; l < 8; ++l) row_sum += acc[l];
        for (; i < cols; ++i) row_sum += (float)rw[i] * x[i];
        put_y(y, row_base + r, row_sum * d.scale + d.bias, accumulate);
    }
}

/* src/chpe_engine.zig:409-436 gemvTileF16 and :439-466 gemvTileF32 */
void oracle_gemv_tile_f16(const uint8_t *cell, const float *x, float *y, size_t row_base, int accumulate) {
    tile_dims d = cell_dims(cell);
    const uint8_t *coded = cell + CELL_HDR;
    for (size_t r = 0; r < d.rows; ++r) {
        float s = 0.0f;
        for (size_t c = 0; c < d.cols; ++c) {
            f16 w;
            memcpy(&w, coded + 2 * (r * d.cols + c), 2);
            s += (float)w * x[c];
        }
        put_y(y, row_base + r, s, accumulate);
    }
}
void oracle_gemv_tile_f32(const uint8_t *cell, const float *x, float *y, size_t row_base, int accumulate) {
    tile_dims d = cell_dims(cell);
    const uint8_t *coded = cell + CELL_HDR;
    for (size_t r = 0; r < d.rows; ++r) {
        float s = 0.0f;
        for (size_t c = 0; c < d.cols; ++c) {
            float w;
            memcpy(&w, coded + 4 * (r * d.cols + c), 4);
            s += w * x[c];
        }
        put_y(y, row_base + r, s, accumulate);
    }
}

/* src/chpe_engine.zig:469-488  gemvTilePolymorphic (unknown widths fall back to W2) */
void oracle_gemv_tile_polymorphic(const uint8_t *cell, const float *x, size_t x_len, float *y, size_t row_base,
                                  int accumulate) {
    switch (cell_quant_bits(cell)) {
    case 4: oracle_gemv_tile_w4(cell, x, y, row_base, accumulate); break;
    case 8: oracle_gemv_tile_w8(cell, x, y, row_base, accumulate); break;
    case 16: oracle_gemv_tile_f16(cell, x, y, row_base, accumulate); break;
    case 32: oracle_gemv_tile_f32(cell, x, y, row_base, accumulate); break;
    default: oracle_gemv_tile_w2(cell, x, x_len, y, row_base, accumulate); break;
    }
}

/* src/qwen72b_engine.zig:119-132  dotTileRow2Bit */
float oracle_dot_tile_row_2bit(const uint8_t *coded, const float *x, size_t x_len, float scale, float bias) {
    float sum = 0.0f;
    for (size_t b = 0; b < x_len / 4; ++b) {
        uint8_t bv = coded[b];
        float w0 = CODEBOOK_W2[bv & 3] * scale + bias;
        float w1 = CODEBOOK_W2[(bv >> 2) & 3] * scale + bias;
        float w2 = CODEBOOK_W2[(bv >> 4) & 3] * scale + bias;
        float w3 = CODEBOOK_W2[(bv >> 6) & 3] * scale + bias;
        size_t base = b * 4;
        sum += w0 * x[base] + w1 * x[base + 1] + w2 * x[base + 2] + w3 * x[base + 3];
    }
    return sum;
}

/* src/qwen72b_engine.zig:135-148  dotTileRow4Bit */
float oracle_dot_tile_row_4bit(const uint8_t *coded, const float *x, size_t x_len, float scale, float bias) {
    float sum = 0.0f;
    for (size_t b = 0; b < x_len / 2; ++b) {
        uint8_t bv = coded[b];
        float w0 = (float)((int)(bv & 0x0F) - 8) * scale + bias;
        float w1 = (float)((int)((bv >> 4) & 0x0F) - 8) * scale + bias;
        sum += w0 * x[2 * b] + w1 * x[2 * b + 1];
    }
    return sum;
}

/* ------------------------------------------------------------------------ */
/* Quantizers                                                               */
/* ------------------------------------------------------------------------ */

/* scripts/pack_qwen72b_chpe.py:138-148  quantize_4bit_block.  blk is [n_blocks,128]
 * f32; np.round is round-half-even (nearbyintf); fp16 casts are RNE.
 * Writes n_blocks*64 packed bytes and n_blocks fp16 scales (as uint16 bits). */
void oracle_quantize_4bit_block(const float *blk, size_t n_blocks, uint8_t *packed, uint16_t *scales) {
    for (size_t bi = 0; bi < n_blocks; ++bi) {
        const float *w = blk + bi * 128;
        float m = 0.0f;
        for (int i = 0; i < 128; ++i) m = fmaxf(m, fabsf(w[i]));
        f16 s = (f16)((m > 1e-8f) ? m / 7.0f : 1.0f);
        float s32 = (s > (f16)1e-8f) ? (float)s : 1.0f;
        for (int i = 0; i < 128; i += 2) {
            float q0 = fminf(fmaxf(nearbyintf(w[i] / s32), -8.0f), 7.0f);
            float q1 = fminf(fmaxf(nearbyintf(w[i + 1] / s32), -8.0f), 7.0f);
            uint8_t n0 = (uint8_t)((int)q0 + 8), n1 = (uint8_t)((int)q1 + 8);
            packed[bi * 64 + i / 2] = (uint8_t)((n0 & 0x0F) | ((n1 & 0x0F) << 4));
        }
        memcpy(&scales[bi], &s, 2);
    }
}

/* scripts/pack_qwen72b_chpe.py:110-135  quantize_2bit_block (codebook
 * 0:0, 1:+1, 2:-2, 3:-1; c0 in bits 1:0 ... c3 in bits 7:6) */
void oracle_quantize_2bit_block(const float *blk, size_t n_blocks, uint8_t *packed, uint16_t *scales) {
    for (size_t bi = 0; bi < n_blocks; ++bi) {
        const float *w = blk + bi * 128;
        float m = 0.0f;
        for (int i = 0; i < 128; ++i) m = fmaxf(m, fabsf(w[i]));
        f16 s = (f16)((m > 1e-8f) ? m / 2.0f : 1.0f);
        float s32 = (s > (f16)1e-8f) ? (float)s : 1.0f;
        for (int i = 0; i < 128; i += 4) {
            uint8_t byte = 0;
            for (int j = 0; j < 4; ++j) {
                float v = w[i + j] / s32;
                uint8_t q = (v >= 0.5f) ? 1 : (v >= -0.5f) ? 0 : (v >= -1.5f) ? 3 : 2;
                byte |= (uint8_t)((q & 3) << (2 * j));
            }
            packed[bi * 32 + i / 4] = byte;
        }
        memcpy(&scales[bi], &s, 2);
    }
}

/* Grouped asymmetric quantizer for the unsigned-code formats (4-bit / 2-bit,
 * group g along K, fp16 scale + fp16 zero-point).  This project's
 * specification (the reference has no such quantizer):
 *   s = fp16((max-min)/(2^b-1)), or 1 when max-min <= 1e-8
 *   z = fp16(clamp(rint(-min/s), 0, 2^b-1))
 *   c = clamp(rint(w/s) + z, 0, 2^b-1)
 * w is [rows, cols] row-major; codes are one byte per weight (unpacked);
 * scales/zeros are [rows, cols/g] fp16 bits. */
void oracle_quantize_asym(const float *w, size_t rows, size_t cols, int bits, int group, uint8_t *codes,
                          uint16_t *scales, uint16_t *zeros) {
    float qmax = (float)((1 << bits) - 1);
    size_t ng = cols / (size_t)group;
    for (size_t r = 0; r < rows; ++r)
        for (size_t g = 0; g < ng; ++g) {
            const float *v = w + r * cols + g * group;
            float mn = v[0], mx = v[0];
            for (int i = 1; i < group; ++i) {
                mn = fminf(mn, v[i]);
                mx = fmaxf(mx, v[i]);
            }
            float range = mx - mn;
            f16 s = (f16)((range > 1e-8f) ? range / qmax : 1.0f);
            float s32 = (float)s;
            if (!(s32 > 0.0f)) s32 = 1.0f, s = (f16)1.0f;
            float zf = fminf(fmaxf(nearbyintf(-mn / s32), 0.0f), qmax);
            f16 z = (f16)zf;
            for (int i = 0; i < group; ++i) {
                float c = fminf(fmaxf(nearbyintf(v[i] / s32) + zf, 0.0f), qmax);
                codes[r * cols + g * group + i] = (uint8_t)c;
            }
            memcpy(&scales[r * ng + g], &s, 2);
            memcpy(&zeros[r * ng + g], &z, 2);
        }
}

/* Grouped symmetric int8 quantizer (group g along K, fp16 scale, codes in
 * [-127,127]).  This project's specification:
 *   s = fp16(max|w|/127), or 1 when max|w| <= 1e-8;  q = clamp(rint(w/s), -127, 127) */
void oracle_quantize_sym8(const float *w, size_t rows, size_t cols, int group, int8_t *codes, uint16_t *scales) {
    size_t ng = cols / (size_t)group;
    for (size_t r = 0; r < rows; ++r)
        for (size_t g = 0; g < ng; ++g) {
            const float *v = w + r * cols + g * group;
            float m = 0.0f;
            for (int i = 0; i < group; ++i) m = fmaxf(m, fabsf(v[i]));
            f16 s = (f16)((m > 1e-8f) ? m / 127.0f : 1.0f);
            float s32 = (float)s;
            if (!(s32 > 0.0f)) s32 = 1.0f, s = (f16)1.0f;
            for (int i = 0; i < group; ++i) {
                float q = fminf(fmaxf(nearbyintf(v[i] / s32), -127.0f), 127.0f);
                codes[r * cols + g * group + i] = (int8_t)q;
            }
            memcpy(&scales[r * ng + g], &s, 2);
        }
}

/* ------------------------------------------------------------------------ */
/* Grouped dequant-GEMV / GEMM specification                                 */
/* y[m][n] = sum_k w(n,k) * x[m][k], with w(n,k) formed in fp32 as           */
/*   signed int8, fp16 scale:            w = (float)q * s                    */
/*   unsigned codes, fp16 scale + zero:  w = ((float)c - z) * s              */
/* and the sum carried in double.  codes are one byte per weight [N][K].    */
/* x_kind: 0 = f32 [M][K], 1 = bf16 bits [M][K].                             */
/* ------------------------------------------------------------------------ */
static float bf16_to_f32(uint16_t b) {
    uint32_t u = (uint32_t)b << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

void oracle_gemv_grouped(int signed_codes, const uint8_t *codes, const uint16_t *scales, const uint16_t *zeros,
                         int group, size_t N, size_t K, const void *x, int x_kind, size_t M, float *y) {
    size_t ng = K / (size_t)group;
    float *wrow = (float *)malloc(K * sizeof(float));
    float *xf = (float *)malloc(M * K * sizeof(float));
    for (size_t i = 0; i < M * K; ++i)
        xf[i] = x_kind == 0 ? ((const float *)x)[i] : bf16_to_f32(((const uint16_t *)x)[i]);
    for (size_t n = 0; n < N; ++n) {
        for (size_t g = 0; g < ng; ++g) {
            f16 s16, z16 = (f16)0.0f;
            memcpy(&s16, &scales[n * ng + g], 2);
            if (zeros) memcpy(&z16, &zeros[n * ng + g], 2);
            float s = (float)s16, z = (float)z16;
            for (int i = 0; i < group; ++i) {
                size_t k = g * group + i;
                uint8_t c = codes[n * K + k];
                wrow[k] = signed_codes ? (float)(int8_t)c * s : ((float)c - z) * s;
            }
        }
        for (size_t m = 0; m < M; ++m) {
            double acc = 0.0;
            for (size_t k = 0; k < K; ++k) acc += (double)wrow[k] * (double)xf[m * K + k];
            y[m * N + n] = (float)acc;
        }
    }
    free(wrow);
    free(xf);
}

/* Threaded variant of oracle_gemv_grouped for the CPU baseline timing: rows
 * are split into contiguous slices over num_workers threads as in
 * src/engine.zig:188-192. */
typedef struct {
    int signed_codes; const uint8_t *codes; const uint16_t *scales, *zeros; int group;
    size_t N, K; const void *x; int x_kind; size_t M; float *y; size_t r0, r1;
} grouped_job;

static void *grouped_thread(void *p) {
    grouped_job *j = (grouped_job *)p;
    size_t ng = j->K / (size_t)j->group;
    size_t rows = j->r1 - j->r0;
    if (rows == 0) return NULL;
    float *ys = (float *)malloc(j->M * rows * sizeof(float));
    oracle_gemv_grouped(j->signed_codes, j->codes + j->r0 * j->K, j->scales + j->r0 * ng,
                        j->zeros ? j->zeros + j->r0 * ng : NULL, j->group, rows, j->K, j->x, j->x_kind, j->M, ys);
    for (size_t m = 0; m < j->M; ++m) memcpy(j->y + m * j->N + j->r0, ys + m * rows, rows * sizeof(float));
    free(ys);
    return NULL;
}

void oracle_gemv_grouped_mt(int signed_codes, const uint8_t *codes, const uint16_t *scales, const uint16_t *zeros,
                            int group, size_t N, size_t K, const void *x, int x_kind, size_t M, float *y,
                            int num_workers) {
    if (num_workers < 1) num_workers = 1;
    if (num_workers > 256) num_workers = 256;
    grouped_job jobs[256];
    pthread_t th[256];
    size_t per = N / (size_t)num_workers;
    for (int w = 0; w < num_workers; ++w) {
        grouped_job j = {signed_codes, codes, scales, zeros, group, N, K, x, x_kind, M, y,
                         (size_t)w * per, (w == num_workers - 1) ? N : (size_t)(w + 1) * per};
        jobs[w] = j;
    }
    for (int w = 1; w < num_workers; ++w) pthread_create(&th[w], NULL, grouped_thread, &jobs[w]);
    grouped_thread(&jobs[0]);
    for (int w = 1; w < num_workers; ++w) pthread_join(th[w], NULL);
}

/* src/engine.zig:1098-1110  computeArgmax (first index of the maximum) */
uint32_t oracle_argmax(const float *logits, size_t n, float *max_out) {
    float mv = -INFINITY;
    uint32_t am = 0;
    for (size_t i = 0; i < n; ++i)
        if (logits[i] > mv) {
            mv = logits[i];
            am = (uint32_t)i;
        }
    if (max_out) *max_out = mv;
    return am;
}
