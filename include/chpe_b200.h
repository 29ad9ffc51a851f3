/*
 * chpe_b200.h -- C ABI of the B200 (sm_100a) quantized dequant-matmul library.
 *
 * Drop-in replacement for the CHPE engine's CPU GEMV operator layer.  Every
 * entry point returns an int status (0 = OK, negative CHPE_E* on error) and
 * never aborts the process; chpe_last_error_string() describes the last error
 * of a context.  Signatures use plain pointers and sizes only.
 *
 * Pointer rules.  Functions with a `_parallel` / `_tile_` name mirror the
 * reference's Zig operators and take HOST pointers, exactly as the reference
 * does: activations are copied to the device, the kernel runs, the result is
 * copied back before the call returns.  Weight pointers passed to them are
 * looked up in the context's registry (chpe_register_*): a registered host
 * weight pointer is served from its resident device copy; an unregistered one
 * is uploaded on first use and cached under that pointer.  The cache checks
 * the shape and a content fingerprint (every byte of a cell; the first and
 * last 4 KiB plus 64 strided windows of a weight matrix), so a host buffer
 * freed and reused for other weights at the same address is re-uploaded;
 * weights modified in place inside the sampled-out bytes must be
 * re-registered with chpe_register_i8.  Functions with a
 * `_dev` suffix take DEVICE pointers and a cudaStream_t (passed as void*) and
 * are asynchronous.
 *
 * Thread safety: calls on one context are serialised by the caller (one
 * context per thread or stream), as the reference's single caller thread is
 * (src/engine.zig:174).
 */
#ifndef CHPE_B200_H
#define CHPE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------- */
enum {
    CHPE_OK = 0,
    CHPE_EINVAL = -1,   /* bad argument (size, format, null pointer)          */
    CHPE_EALIGN = -2,   /* pointer or size misaligned for the device layout   */
    CHPE_ENOMEM = -3,   /* device or host allocation failed                   */
    CHPE_ECUDA = -4,    /* CUDA runtime error                                 */
    CHPE_ETIMEOUT = -5, /* a kernel's bounded wait expired (error flag set)   */
    CHPE_ENOTSUP = -6,  /* combination not supported                          */
    CHPE_ENOENT = -7    /* handle / registered pointer not found              */
};

/* ---- formats ------------------------------------------------------------ */
/* How the stored codes map to weight values.  `bits` is 2, 4 or 8; codes are
 * packed row-major, K contiguous, least-significant bits first inside each
 * byte (element 2i in the low nibble of byte i for 4-bit; element 4i in bits
 * 1:0 for 2-bit).  That is the reference packer's byte order
 * (scripts/pack_qwen72b_chpe.py:138-148, :110-135) and also little-endian
 * uint32 packing. */
enum {
    /* int8 codes, one fp32 scale per tensor; activations int8 (W8A8).
     * src/tensor_map.zig:7-51 scales, src/engine.zig:227-251 gemvParallel. */
    CHPE_SCHEME_I8_TENSOR = 1,
    /* signed int8 codes, fp16 scale per group:  w = q * s[n, k/group] */
    CHPE_SCHEME_I8_GROUP_F16 = 2,
    /* unsigned codes, fp16 scale + fp16 zero per group: w = (c - z) * s */
    CHPE_SCHEME_U_GROUP_F16_ZERO = 3,
    /* unsigned codes, fp16 scale per group, constant zero-point `zero`:
     * w = (c - zero) * s.  zero = 8 is the reference's offset-8 int4 with
     * group-128 scales (src/kernels/cuda/bench_t4_qwen35.cu:24-87). */
    CHPE_SCHEME_U_GROUP_F16_CONST_ZERO = 4,
    /* the reference 2-bit codebook {0:0, 1:+1, 2:-2, 3:-1} with fp16 group
     * scales: w = LUT[c] * s  (src/chpe_engine.zig:216-286) */
    CHPE_SCHEME_W2_CODEBOOK_GROUP_F16 = 5,
    /* per-row fp32 affine: w = value(c) * scale[n] + offset[n] summed per
     * weight, plus bias[n] added once per row; value(c) is the signed int8,
     * offset-8 nibble or 2-bit codebook value.  Covers the per-tile
     * scale/bias cells (src/chpe_engine.zig:319-406). */
    CHPE_SCHEME_ROW_AFFINE_F32 = 6
};

/* activation dtypes */
enum { CHPE_X_F32 = 0, CHPE_X_BF16 = 1, CHPE_X_F16 = 2, CHPE_X_I8 = 3 };

typedef struct chpe_fmt {
    int32_t bits;   /* 2, 4, 8                                                */
    int32_t scheme; /* CHPE_SCHEME_*                                          */
    int32_t group;  /* group size along K; 0 means one group per row (= K)     */
    float zero;     /* constant zero-point for CHPE_SCHEME_U_GROUP_F16_CONST_ZERO */
} chpe_fmt;

typedef struct chpe_ctx chpe_ctx;
typedef struct chpe_tensor chpe_tensor;

/* ---- context ------------------------------------------------------------ */
int chpe_init(int device, chpe_ctx **out);
int chpe_destroy(chpe_ctx *ctx);
const char *chpe_last_error_string(const chpe_ctx *ctx);
/* Library build/version string (no context needed). */
const char *chpe_version(void);
/* Kernels this library has launched in this process so far (all contexts).
 * A launch recorded into a CUDA graph counts once, at capture. */
unsigned long long chpe_kernel_launches(void);
/* Device sync + read-back of the kernels' error flag (bounded waits that
 * expired); returns CHPE_ETIMEOUT if any kernel recorded one. */
int chpe_sync(chpe_ctx *ctx);

/* ---- weight upload (the operator surface's tiles become device tensors) --- */
/* Upload a [rows, cols] matrix given as packed codes plus its scales.
 *   codes:  rows * row_stride bytes (row_stride >= cols*bits/8), host or device
 *   scales: per scheme -- fp16 [rows, cols/group]; fp32 [1] (I8_TENSOR);
 *           fp32 [rows] (ROW_AFFINE_F32)
 *   zeros:  fp16 [rows, cols/group] (U_GROUP_F16_ZERO) or fp32 offsets [rows]
 *           (ROW_AFFINE_F32), else NULL
 *   bias:   fp32 [rows] added once per output row, or NULL
 * Pointers may be host or device memory (detected).  The device copy is
 * repacked into the strip layout and owned by the context.  Device inputs are
 * read on the context's stream: work on other streams that writes them must
 * be complete before the call.  The call returns after the repack finished.
 * Replaces: archive.getTileU16Direct(lmap.*_tile) + the per-tensor scales of
 * LayerTensorMap (src/engine.zig:609-612, src/tensor_map.zig:7-51). */
int chpe_upload_matrix(chpe_ctx *ctx, const chpe_fmt *fmt, const void *codes, size_t row_stride, const void *scales,
                       const void *zeros, const float *bias, size_t rows, size_t cols, chpe_tensor **out);

/* Upload a run of CHPE cells (17408-byte Cell = 64 B header + 16384 B codes +
 * 960 B payload, src/geometry.zig:243-256) found every `tile_stride` bytes
 * starting at `first_cell` (20480 for standard archives, 17408 for dense).
 * Each cell contributes TileDims.rows rows of TileDims.cols columns; all cells
 * must share quant_bits, cols and the group-128 flag.  Semantics per cell
 * follow gemvTileW2/W4/W8 (src/chpe_engine.zig:219-406), including the
 * group-128 scales and 8 fp16 outlier columns of 2-bit cells. */
int chpe_upload_cells(chpe_ctx *ctx, const void *first_cell, size_t n_cells, size_t tile_stride, chpe_tensor **out);

/* Grouped quantizer on the device (this library's packer; the reference has
 * none for these formats): fp32 w [rows, cols] -> one code byte per weight
 * [rows, cols] plus fp16 scales (and zeros) [rows, cols/group].
 *   symmetric != 0: s = fp16(max|w|/127), q = clamp(rint(w/s), -127, 127)
 *   symmetric == 0: s = fp16((max-min)/(2^bits-1)), z = fp16(clamp(rint(-min/s))),
 *                   c = clamp(rint(w/s) + z, 0, 2^bits-1)
 * All pointers are device pointers; asynchronous on `stream`. */
int chpe_quantize_group_dev(chpe_ctx *ctx, const float *w, size_t rows, size_t cols, int bits, int group,
                            int symmetric, uint8_t *codes, uint16_t *scales, uint16_t *zeros, void *stream);

int chpe_tensor_free(chpe_ctx *ctx, chpe_tensor *t);
/* rows / cols / bits of a tensor and its device bytes (codes + metadata). */
int chpe_tensor_info(const chpe_tensor *t, size_t *rows, size_t *cols, int *bits, size_t *device_bytes);

/* Read a resident tensor back out of the device layout, bit for bit as it
 * was uploaded: codes row-major [rows][ceil(cols*bits/8)] bytes packed least
 * significant bits first (signed int8, offset-8 nibbles, 2-bit codebook codes
 * or unsigned codes, as given to the upload), scales as fp16 [rows][groups]
 * (fp32 [rows] for per-row affine cells; nothing for the per-tensor W8A8
 * scale), zeros as fp16 [rows][groups] (scale + zero tensors only; else NULL).
 * Host or device destination pointers; synchronous.  No counterpart in the
 * reference (its weights never leave their host layout); it exists to show
 * that the device repack is lossless. */
int chpe_tensor_unpack(chpe_ctx *ctx, const chpe_tensor *t, void *codes, void *scales, void *zeros);

/* Register a host weight region as the source of later `_parallel` calls.
 * Replaces the mmap'd archive handed to the engine (src/weight_archive.zig:173-211):
 * the shim registers each int8 weight tensor once at init. */
int chpe_register_i8(chpe_ctx *ctx, const int8_t *host_weights, size_t rows, size_t cols);

/* ---- GEMV on resident tensors (device pointers, async on `stream`) ------- */
/* y[M, rows] = x[M, cols] . W^T for M = 1..64 activation rows.
 *   x: x_dtype CHPE_X_F32/BF16/F16, or CHPE_X_I8 with per-row scales
 *      x_scales[M] (W8A8: y = float(sum q_w q_x) * (scale_w * x_scales[m]))
 *   accumulate != 0 adds into y (gemvTile* `accumulate`, src/chpe_engine.zig:310-314) */
int chpe_gemv_dev(chpe_ctx *ctx, const chpe_tensor *w, const void *x, int x_dtype, const float *x_scales, int M,
                  float *y, int accumulate, void *stream);
/* mlp_out[M, rows] = silu(x.Wg^T) * (x.Wu^T), one pass over both weights.
 * Replaces gemvGateUpSwiGLUParallel (src/engine.zig:285-313). */
int chpe_gemv_gateup_swiglu_dev(chpe_ctx *ctx, const chpe_tensor *gate, const chpe_tensor *up, const void *x,
                                int x_dtype, const float *x_scales, int M, float *mlp_out, void *stream);
/* Activation fragments shared by several GEMVs that read the same input (the
 * Q/K/V projections, gate/up, the Gated-DeltaNet in-projections read one
 * normalised hidden state: src/engine.zig:615-617, :641-642).  The reference
 * quantizes x once and passes the int8 vector to each gemvParallel; here x is
 * converted once into the MMA operand layout (fp16 pairs plus block sums, or
 * int8 with per-row scales) and each GEMV streams only its weights.
 *   create: M = 1..8 rows of `like`'s cols; any tensor with the same cols,
 *           code layout and epilogue block (same bits / group) can consume it
 *   fill:   x [M, cols] device pointer of x_dtype (int8 needs x_scales[M];
 *           fp32 into an int8 weight runs the reference's dynamic quantizer) */
typedef struct chpe_xfrag chpe_xfrag;
int chpe_xfrag_create(chpe_ctx *ctx, const chpe_tensor *like, int M, int x_dtype, chpe_xfrag **out);
int chpe_xfrag_fill_dev(chpe_ctx *ctx, chpe_xfrag *xf, const void *x, const float *x_scales, void *stream);
int chpe_gemv_xfrag_dev(chpe_ctx *ctx, const chpe_tensor *w, const chpe_xfrag *xf, float *y, int accumulate,
                        void *stream);
int chpe_gemv_gateup_swiglu_xfrag_dev(chpe_ctx *ctx, const chpe_tensor *gate, const chpe_tensor *up,
                                      const chpe_xfrag *xf, float *mlp_out, void *stream);
/* ys[r][M, rows_r] = x . W_r^T for n = 1..4 tensors of the same cols and format
 * in ONE launch (the Q, K, V projections, src/engine.zig:615-617, or the
 * Gated-DeltaNet in-projections, :641-642, which the reference runs as
 * separate gemvParallel calls on the same quantized x). */
int chpe_gemv_multi_xfrag_dev(chpe_ctx *ctx, int n, const chpe_tensor *const *ws, const chpe_xfrag *xf,
                              float *const *ys, void *stream);
int chpe_xfrag_free(chpe_ctx *ctx, chpe_xfrag *xf);

/* Fill fragments from one of the step's elementwise producers, fused into the
 * fill (one kernel instead of producer + fill; the producer's output never
 * reaches memory).  M rows of `cols` values (the fragment's K):
 *   CHPE_XOP_PLAIN      x[m][k] of x_dtype (as chpe_xfrag_fill_dev)
 *   CHPE_XOP_RMSNORM    x[m][k] * 1/sqrt(mean_k(x[m]^2) + eps) * aux[k]
 *                       (rmsnorm, src/kernels/neon.zig:673-702; aux = gamma)
 *   CHPE_XOP_SILU_MUL   silu(x[m][k]) * aux[m][k]  (siluMul, neon.zig:705-712)
 *   CHPE_XOP_ATTN_STUB  x[m][k % kv_dim], or head-aligned with head_dim/group
 *                       (full-attention stand-in, src/engine.zig:619-623)
 *   CHPE_XOP_SSM_STUB   q = x[m][k % qkv_dim], z = aux[m][k]: q * silu(z), or
 *                       silu(q) * z when silu_on_qkv (Gated-DeltaNet stand-in,
 *                       src/engine.zig:651-654 / :813 / :988)
 * Row strides ldx / ld_aux are in elements; every op other than PLAIN reads
 * fp32.  RMSNorm's gamma is treated like a weight: the fill may read it
 * before the kernel ahead of it on the stream has finished, so that kernel
 * must not write it.  No counterpart in the reference, whose engine
 * materialises each producer's output before quantizing it for the next
 * gemvParallel. */
#define CHPE_XOP_PLAIN 0
#define CHPE_XOP_RMSNORM 1
#define CHPE_XOP_SILU_MUL 2
#define CHPE_XOP_ATTN_STUB 3
#define CHPE_XOP_SSM_STUB 4
typedef struct chpe_xsrc {
    int op;
    const void *x;
    int x_dtype; /* CHPE_XOP_PLAIN only */
    int ldx;
    const float *aux;
    int ld_aux;
    float eps;
    int kv_dim, head_dim, group; /* CHPE_XOP_ATTN_STUB */
    int qkv_dim, silu_on_qkv;    /* CHPE_XOP_SSM_STUB */
} chpe_xsrc;
int chpe_xfrag_fill_op_dev(chpe_ctx *ctx, chpe_xfrag *xf, const chpe_xsrc *src, void *stream);
/* GEMV with the producer fused into it: every CTA builds the activation
 * fragments of its own K-slice from `src` (fp32 rows; RMSNorm statistics
 * computed in the CTA), so no fill kernel or fragment buffer sits between two
 * GEMVs.  mode 0: ys[r][M, rows_r] (+)= x . W_r^T for n = 1..4 tensors of the
 * same cols and format (accumulate != 0 adds into y); mode 1: n = 2 (gate,
 * up), ys[0] = silu(x.Wg^T) * (x.Wu^T).  fp16-path tensors only (not W8A8),
 * M = 1..8.  Same results as chpe_xfrag_fill_op_dev + the _xfrag_ GEMVs. */
int chpe_gemv_src_dev(chpe_ctx *ctx, int mode, int n, const chpe_tensor *const *ws, const chpe_xsrc *src, int M,
                      float *const *ys, int accumulate, void *stream);

/* Prefill dequant-GEMM on the 5th-generation tensor cores (tcgen05, fp32
 * accumulation in tensor memory): y[M, rows] (+)= x[M, cols] . dequant(W)^T
 * for any M >= 1 (efficient from M = 64 up; tiles of 128 rows).
 *   x: CHPE_X_BF16 / F16 / F32 device rows [M][cols], converted once to fp16
 *      (bf16 and fp16 exactly); W is dequantized in shared memory to fp16
 *      w = fp16(q * s) or fp16((c - z) * s) and never written back to HBM
 *   W: the same resident tensor the GEMVs use; 8-bit with an fp16 scale per
 *      32 columns (CHPE_SCHEME_I8_GROUP_F16, group 32), or 4-bit with fp16
 *      scale (+ zero) per 64k columns (U_GROUP_F16_ZERO / _CONST_ZERO);
 *      other formats return CHPE_ENOTSUP
 *   y: fp32 rows [M][ldy] (ldy >= rows); accumulate != 0 adds into y
 * No counterpart in the reference, whose engine runs every prompt token
 * through the batch-1 step (src/main.zig:175-195). */
int chpe_gemm_prefill_dev(chpe_ctx *ctx, const chpe_tensor *w, const void *x, int x_dtype, int M, float *y,
                          int ldy, int accumulate, void *stream);

/* ---- tensor parallelism: one-shot all-reduce over NVLink peer memory ------
 * hidden[i] += sum over the `world` ranks of part_r[i], i < n, after the O and
 * down projections of a tensor-parallel block.  Each rank stores its partial
 * into every peer's receive area (P2P stores through CUDA IPC mappings), each
 * value tagged with the exchange's epoch in the same 64-bit word, polls its
 * own area until every peer's values carry the epoch (bounded: 1 s, then
 * CHPE_ETIMEOUT at chpe_sync) and sums the partials in rank order -- identical
 * bits on every rank.  One kernel, one NVLink trip, no NCCL on this path.
 * Setup: chpe_comm_create on every rank, exchange the chpe_comm_handle_bytes()
 * handle of every rank (any host transport), chpe_comm_open_peers with all
 * ranks' handles in rank order.  Every rank must issue the same sequence of
 * exchanges.  No counterpart in the single-process reference. */
typedef struct chpe_comm chpe_comm;
int chpe_comm_create(chpe_ctx *ctx, int world, int rank, size_t max_elems, chpe_comm **out);
size_t chpe_comm_handle_bytes(void);
int chpe_comm_handle(const chpe_comm *comm, void *out);
int chpe_comm_open_peers(chpe_comm *comm, const void *handles);
int chpe_allreduce_residual_dev(chpe_comm *comm, const float *part, float *hidden, size_t n, void *stream);
/* The vocabulary-split LM head's argmax over the ranks: on entry idx[m] and
 * maxv[m] (m < M <= 32, device memory) hold row m's argmax within this rank's
 * shard (index local to the shard) and its value; on return every rank holds
 * the global pair -- index_base (the shard's first vocabulary row) is added
 * to the local index, then the largest value wins and ties go to the smaller
 * global index, the rule of src/engine.zig:1098-1110 computeArgmax.  Same
 * exchange (tagged pushes, bounded waits, failure mark) as the all-reduce, in
 * the same ordered sequence of exchanges on every rank.  Replaces an
 * all-gather of the pairs; no counterpart in the single-process reference. */
int chpe_argmax_merge_dev(chpe_comm *comm, int *idx, float *maxv, int M, int index_base, void *stream);
/* The all-reduce fused with the fill that consumes it: hidden[m][:] += the
 * sum over ranks of part_r[m][:] for the fragments' M rows of K columns (rows
 * contiguous, stride K), then xf is filled with RMSNorm(hidden) * gamma --
 * the same bits as chpe_allreduce_residual_dev followed by
 * chpe_xfrag_fill_op_dev(CHPE_XOP_RMSNORM of hidden), in one kernel: each
 * fill CTA exchanges its own columns.  CHPE_ENOTSUP (nothing launched) for
 * fragments with outliers or int8 operands, or rows that do not fit; the
 * caller then runs the two calls.  Same exchange sequence rule as the
 * all-reduce; no counterpart in the single-process reference. */
int chpe_allreduce_fill_dev(chpe_comm *comm, const float *part, float *hidden, chpe_xfrag *xf, const float *gamma,
                            float eps, int pushed, void *stream);
/* The O / down projection of a tensor-parallel block with its half of the
 * exchange built in: y[m][:] = xf . W^T (M rows of W's row count, stride
 * that count) as chpe_gemv_xfrag_dev, and every finished output is also
 * stored, tagged with the exchange's epoch, into every peer's receive area
 * by the GEMV's own CTAs, overlapped with the weight streaming.  The very
 * next exchange on `comm` must then be chpe_allreduce_fill_dev(part = y,
 * pushed = 1), which only collects and sums.  (pushed = 0: the fill sends
 * the partials itself.)  No counterpart in the single-process reference. */
int chpe_gemv_xfrag_push_dev(chpe_ctx *ctx, const chpe_tensor *w, const chpe_xfrag *xf, float *y, chpe_comm *comm,
                             void *stream);
/* A comm object whose bounded wait expired is failed: the ranks' epochs may
 * be out of step, so every later chpe_allreduce_residual_dev on it returns
 * CHPE_ETIMEOUT at once (and a launch already queued, e.g. inside a CUDA
 * graph, skips the exchange and records the error for chpe_sync) until
 * chpe_comm_reset.  chpe_comm_failed returns 1 when failed, 0 when not.
 * chpe_comm_reset waits for the device, then clears this rank's epochs, slots
 * and failed mark; call it on EVERY rank between two host barriers (no rank
 * may issue an all-reduce before all ranks have reset). */
int chpe_comm_failed(const chpe_comm *comm);
int chpe_comm_reset(chpe_comm *comm);
int chpe_comm_destroy(chpe_comm *comm);

/* Dynamic per-row int8 activation quantization (device): for each of M rows of
 * length n: s = max|x|/127 (1 if max <= 1e-9), q = clamp(round_half_away(x/s))
 * -- src/kernels/neon.zig:644-670 quantizeActivationInt8, bit-exact. */
int chpe_quantize_act_i8_dev(chpe_ctx *ctx, const float *x, int M, size_t n, int8_t *q, float *scales,
                             void *stream);

/* ---- the rest of a decode / verify step (device pointers, async) --------
 * The reference's Qwen35Engine.step orchestration (src/engine.zig:567-734,
 * stepBatch4 :753-900, stepBatch8 :902-1095) around the GEMVs.  Rows are
 * [M][dim] contiguous.  The residual adds of the engine are done by the GEMV
 * itself (chpe_gemv_dev with accumulate = 1 into the hidden state). */
/* src/engine.zig:567-580 embedToken: out[m][i] = table[tokens[m]][i] * scale */
int chpe_embed_i8_dev(chpe_ctx *ctx, const int8_t *table, float scale, int hidden, int vocab, const int *tokens,
                      int M, float *out, void *stream);
/* src/kernels/neon.zig:673-702 rmsnorm: y = x * (1/sqrt(mean(x^2)+eps)) * gamma */
int chpe_rmsnorm_dev(chpe_ctx *ctx, const float *x, const float *gamma, int M, int n, float eps, float *y,
                     void *stream);
/* src/engine.zig:619-623 full-attention stand-in: out[i] = v[i % kv_dim] when
 * head_dim == 0; else head-aligned (query head h of head_dim columns takes kv
 * head h / group), which shards with the heads under tensor parallelism */
int chpe_mix_attn_stub_dev(chpe_ctx *ctx, const float *v, int kv_dim, int M, int out_dim, int head_dim, int group,
                           float *out, void *stream);
/* src/engine.zig:651-654 Gated-DeltaNet stand-in: out[i] = qkv[i % qkv_dim] * silu(z[i]);
 * with silu_on_qkv (stepBatch4/8, src/engine.zig:813, :988): out[i] = silu(qkv[i]) * z[i] */
int chpe_mix_ssm_stub_dev(chpe_ctx *ctx, const float *qkv, int qkv_dim, const float *z, int z_dim, int M,
                          int out_dim, int silu_on_qkv, float *out, void *stream);
/* src/kernels/neon.zig:705-712 siluMul */
int chpe_silu_mul_dev(chpe_ctx *ctx, const float *g, const float *u, size_t n, float *out, void *stream);
/* src/engine.zig:1098-1110 computeArgmax (first index of the maximum), per row */
int chpe_argmax_dev(chpe_ctx *ctx, const float *logits, int M, int n, int *idx, float *maxv, void *stream);

/* ---- token mixers (device pointers, async) ---------------------------------
 * Rows of a step are consecutive positions of one sequence: row m is at
 * position *pos + m, where *pos (a device int) counts the positions already
 * cached; chpe_pos_advance_dev(pos, M) moves it on after the step.
 *
 * Grouped-query decode attention with rotary position embeddings and a KV
 * cache -- applyRope (src/qwen72b_engine.zig:90-111, src/chpe_engine.zig:191-212),
 * the KV-cache update and the GQA softmax attention of forwardDecode
 * (src/qwen72b_engine.zig:291-369, src/chpe_engine.zig:690-745):
 *   q [M][ldq]: per q head head_dim values (followed by head_dim output-gate
 *     values when gated: out = attn * sigmoid(gate), the Qwen3.5 layout)
 *   k, v [M][ldkv]: kv_heads x head_dim values of the new positions
 *   kcache, vcache: this layer's fp32 [max_seq][kv_heads][head_dim]; the
 *     rotated keys and the values of the step's positions are written there
 *   out [M][ldo]: q_heads x head_dim
 * RoPE pairs element i with i + head_dim/2, angle = p / theta^(2i/head_dim);
 * scores are scaled by 1/sqrt(head_dim); query head h reads kv head
 * h / (q_heads / kv_heads).  M <= 8, head_dim <= 256, (q_heads / kv_heads) * M
 * <= 64.  A step past max_seq records an error (chpe_sync) and writes nothing.
 * The RoPE factors are tabulated per (theta, head_dim, max_seq) in the
 * context on first use (that first call synchronises the stream, so it must
 * come before any stream capture); two launches: per kv head and split of 64
 * positions the partial softmax, then per query head the combination. */
int chpe_attn_decode_dev(chpe_ctx *ctx, const float *q, int ldq, const float *k, const float *v, int ldkv,
                         float *kcache, float *vcache, const int *pos, int M, int q_heads, int kv_heads,
                         int head_dim, int max_seq, float rope_theta, int gated, float *out, int ldo, void *stream);
/* Gated-DeltaNet linear attention with its causal conv1d -- Conv1DRingBuffer
 * step / convolve and LinearAttentionState.update (src/ssm.zig:11-99):
 *   qkv [M][ldqkv]: channels q (heads x key_dim), k (heads x key_dim),
 *     v (heads x value_dim) of the step's rows (the in-projection's output)
 *   conv_w [C][4]: per channel, tap j weighs the input j positions back
 *     (C = heads * (2 key_dim + value_dim))
 *   ring [16][C]: inputs of earlier positions (slot = position % 16), updated
 *   state [heads][key_dim][value_dim] fp32, updated; decay [heads]
 *   out [M][ldo]: y = q S per head (heads x value_dim)
 * Per row, in order: conv over the last 4 inputs of each channel, then
 * S = decay[h] * S + k^T v and y = q S.  key_dim 128, value_dim a multiple
 * of 32, M <= 8. */
int chpe_deltanet_step_dev(chpe_ctx *ctx, const float *qkv, int ldqkv, const float *conv_w, float *ring,
                           float *state, const float *decay, const int *pos, int M, int heads, int key_dim,
                           int value_dim, float *out, int ldo, void *stream);
/* *pos += M on the device (after a step's mixers). */
int chpe_pos_advance_dev(chpe_ctx *ctx, int *pos, int M, void *stream);

/* Allocation-free variant of chpe_gemv_dev (plain GEMV, M = 1..8).  No
 * counterpart in the reference.  For callers that cannot allocate device
 * memory when they run a GEMV: host engines that reserve all the device
 * memory they will ever use once at start-up (one arena, sized next to the
 * other jobs on a shared GPU) and treat any later cudaMalloc as a failure, and
 * latency-critical decode loops that cannot afford cudaMalloc's implicit
 * device synchronisation.  chpe_gemv_dev may grow the context's scratch with
 * cudaMalloc; this function never calls cudaMalloc, cudaFree or any
 * allocating routine.  Its scratch is one static device array of 16 MiB that
 * every GPU loading the library holds until the process exits; a shape whose
 * scratch needs more returns CHPE_EINVAL with the required size.  All calls
 * share that array and it keeps the last call's contents (its arrival and
 * work counters are cleared with a memset at the start of every call), so
 * calls that overlap on the GPU race.
 * The first call on each device (and the first after the device's context was
 * destroyed and re-created, e.g. by cudaDeviceReset) looks up the array's
 * device address with that device current; make that first call before any
 * stream capture. */
int chpe_gemv_noalloc_dev(chpe_ctx *ctx, const chpe_tensor *w, const void *x, int x_dtype, const float *x_scales,
                          int M, float *y, void *stream);

/* ---- reference-shaped host-pointer operators (synchronous) --------------- */
/* src/engine.zig:227-251 gemvParallel(weights, scale_w, x_q8, scale_x, rows, cols, out) */
int chpe_gemv_parallel(chpe_ctx *ctx, const int8_t *weights, float scale_w, const int8_t *x_q8, float scale_x,
                       size_t rows, size_t cols, float *out);
/* src/engine.zig:285-313 gemvGateUpSwiGLUParallel(gate, sg, up, su, x_q8, sx, rows, cols, mlp_out) */
int chpe_gemv_gate_up_swiglu_parallel(chpe_ctx *ctx, const int8_t *gate_weights, float scale_gate,
                                      const int8_t *up_weights, float scale_up, const int8_t *x_q8, float scale_x,
                                      size_t rows, size_t cols, float *mlp_out);
/* src/engine.zig:357-391 gemvBatch4Parallel(w, s_w, x0..x3, scales_x[4], rows, cols, out0..out3) */
int chpe_gemv_batch4_parallel(chpe_ctx *ctx, const int8_t *weights, float scale_w, const int8_t *x0,
                              const int8_t *x1, const int8_t *x2, const int8_t *x3, const float scales_x[4],
                              size_t rows, size_t cols, float *out0, float *out1, float *out2, float *out3);
/* src/engine.zig:434-460 gemvBatch8Parallel(w, s_w, x[8], scales_x[8], rows, cols, out[8]) */
int chpe_gemv_batch8_parallel(chpe_ctx *ctx, const int8_t *weights, float scale_w, const int8_t *const x[8],
                              const float scales_x[8], size_t rows, size_t cols, float *const out[8]);
/* src/kernels/neon.zig:644-670 quantizeActivationInt8(x, out_q8) -> scale (host) */
int chpe_quantize_activation_int8(chpe_ctx *ctx, const float *x, size_t n, int8_t *out_q8, float *scale_out);
/* src/chpe_engine.zig:469-488 gemvTilePolymorphic(cell, x, y, row_base, accumulate):
 * x has x_len fp32 values, y is written at y[row_base + r].  Cells with
 * quant_bits 16/32 return CHPE_ENOTSUP. */
int chpe_gemv_tile_polymorphic(chpe_ctx *ctx, const void *cell, const float *x, size_t x_len, float *y,
                               size_t row_base, int accumulate);

#ifdef __cplusplus
}
#endif
#endif /* CHPE_B200_H */
