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
    int n_strips = 0;
    int n_blocks = 0;     // blocks per strip (K padded to whole blocks)
    int span = 0;         // columns per block
    int block_bytes = 0;  // codes + metadata of one block of one strip
    int gpb = 0;          // metadata groups per block
    int gshift = -1;      // log2(group) when group <= span, else -1
    int group = 0;        // columns per group (K when one group per row)
    int n_groups = 0;     // groups per row
    float scale = 1.0f;   // per-tensor scale (S8 layout)
    float zc = 0.0f;      // constant zero-point (kMetaS16)
    uint32_t xorv = 0;    // XOR applied to every stored code (F16 layout: int8 ^ 0x80, 2-bit codebook ^ 2)
    uint8_t *codes = nullptr;  // n_strips * n_blocks * block_bytes
    float *bias = nullptr;
    int *out_cols = nullptr;  // [N][8] outlier columns, -1 = none
    __half *out_w = nullptr;  // [N][8] outlier weights
    size_t bytes = 0;
};

// Where the activations of a fragment fill come from (xfill / xmaterialize):
// the plain rows x, or one of the step's elementwise producers fused in.
enum XSrcOp : int { kXPlain = 0, kXRmsnorm = 1, kXSiluMul = 2, kXAttnStub = 3, kXSsmStub = 4 };
struct XSrc {
    int op = kXPlain;
    const void *x = nullptr;  // rows [M][ldx] (fp32 except for kXPlain)
    int dt = 0;               // kXPlain: CHPE_X_* of x
    int ldx = 0;
    const float *aux = nullptr;  // gamma [K] (rmsnorm), up [M][ld_aux] (silu*mul), z [M][ld_aux] (ssm)
    int ld_aux = 0;
    float eps = 0.0f;
    int kv_dim = 1, head_dim = 0, group = 1;  // attention stand-in
    int qkv_dim = 1, silu_on_qkv = 0;         // Gated-DeltaNet stand-in
};
// Tensor-parallel exchange (comm.cu): the peers' receive areas as
// this rank sees them.
constexpr int kCommMaxRanks = 8;
constexpr int kErrCommWait = 31;
constexpr int kErrCommFailed = 32;  // an exchange issued on a comm object that failed before
struct CommPeers {
    // each rank's receive area [2][world][slot_elems] of tagged words (value
    // bits | epoch << 32): peer mappings, this rank's own one locally
    unsigned long long *tagged[kCommMaxRanks];
};
// An all-reduce of partial sums fused in front of a fragment fill: before the
// fill reads row tok of x (= hidden), each fill CTA sums its columns of the
// ranks' partials [M][K] into hidden (the one-shot all-reduce's exchange and
// arithmetic).  world = 0: none.
struct FillExchange {
    CommPeers peers;
    int world = 0, rank = 0;
    int pushed = 0;  // the partials are in the peers' slots already (a pushing GEMV sent them)
    size_t slot_elems = 0;
    const float *part = nullptr;  // this rank's partials [M][K]
    float *hidden = nullptr;      // [M][K], += the sum of the ranks' partials (the fill's x)
    unsigned *ctr = nullptr;      // epoch, arrival ticket, failed mark
    unsigned *host_failed = nullptr;
    int *err = nullptr;
};

struct GemvSrc {
    const uint8_t *codes;
    const float *bias;
    const int *out_cols;
    const __half *out_w;
    float scale;
    float zc;
};

constexpr int kSG = 4;      // strips per strip group (the GEMV's unit along N)
constexpr int kMaxSrc = 4;  // matrices one plain GEMV launch can cover

struct GemvParams {
    GemvSrc src[kMaxSrc];  // gate/up: src[0] = gate, src[1] = up
    // Plain GEMV: up to kMaxSrc matrices with the same K and format (read from
    // the same activation fragments) concatenated along N, each starting on a
    // strip-group boundary: strip group sg belongs to source r with
    // sg0[r] <= sg < sg0[r + 1] (sg0[r] = INT_MAX past nsrc).
    int nsrc;
    int sg0[kMaxSrc + 1];
    int nstr[kMaxSrc];   // strips of each source
    int rows[kMaxSrc];   // outputs of each source
    float *ys[kMaxSrc];  // y of each source, rows [M][ldys[r]]
    int ldys[kMaxSrc];
    int N, K, M;
    int n_strips, n_blocks, block_bytes, gshift;
    int meta_kind;
    int n_sg;  // strip groups (units along N)
    int n_ks;  // K-slices; CTA b works on slice b % n_ks
    int bpk;   // blocks per K-slice
    // work units: strip groups below n_whole whole per K-slice, the others in
    // chunks of bc blocks; cfull chunks per full K-slice, ctot chunks over the
    // whole K (= workspace slots per strip group); pref static units per CTA
    // when the first units are chunks; the rest are drawn from work_ctr
    int n_whole, bc, cfull, ctot, pref;
    const void *xf;
    const float *xs;
    const float *xe;  // row unscale factors [M] (2^-e of the fill's row scaling); fp16 path
    const float *sx;
    const float *xrow;  // fp32 activations [M][K] (outlier columns), or null
    float *y;
    int ldy;
    int accumulate;
    void *ws;             // chunk sums [n_sg][ctot][kSG * 16 * M]
    unsigned *split_cnt;  // [n_sg] arrivals of chunk sums (self-resetting)
    unsigned *work_ctr;   // [n_ks] work counters (self-resetting)
    int rmode;            // chunk sums: 0 by the last chunk's CTA, 1 by chpe_qgemv_reduce_kernel (set at launch)
    int gk;               // CTAs per K-slice (set at launch)
    int xstream;          // activations stream through the ring with the weights (set at launch)
    int nstages;          // ring stages, 2 or 3 (set at launch)
    // fused fill: with `fused` set, every CTA builds the activation fragments
    // of its K-slice in shared memory from `xsrc` (fp32 rows [M][K]) instead
    // of copying prepared ones (xf / xs unused)
    XSrc xsrc;
    int fused;
    int *err;
    // tensor-parallel push (plain mode): every finished output y[tok][row]
    // also goes, tagged with the comm object's next epoch, into slot
    // [epoch & 1][push.rank] of every peer's receive area at tok * ldy + row;
    // the RMSNorm fill that consumes the exchange then only collects.
    // push.world = 0: none.
    FillExchange push;
};

// Scratch a GEMV call needs, owned by the caller (context).
struct GemvScratch {
    void *xf = nullptr;
    float *xs = nullptr, *sx = nullptr;
    void *ws = nullptr;
    unsigned *counters = nullptr;  // arrival counters (one per strip group), then work counters
    size_t xf_bytes = 0, xs_bytes = 0, sx_bytes = 0, ws_bytes = 0, counters_n = 0;
};

constexpr int kMaxKs = 256;

// Launch plan of one GEMV (computed on the host).
struct GemvPlan {
    int mode = 0;  // 0 plain, 1 gate/up SwiGLU
    int n_sg = 0, n_ks = 0, bpk = 0, grid = 0;
    int n_whole = 0, bc = 1, cfull = 1, ctot = 1, pref = 1;  // work units (GemvParams)
    long items_min = 0;  // units of the shortest K-slice (bound on CTAs per slice)
    int rmode = 0;       // chunk sums: 0 in the GEMV kernel, 1 by a second kernel (more than two rows)
    int xstream = 0;     // 1: activations stream through the ring (more than two rows): no K-slices
    int nstages = 3;     // ring stages
    int sms = 148;
    int e_cols = 0;  // epilogue block (columns)
    bool xsplit = false;
    // activation operand: 0 fp16/bf16, two k-steps per fragment unit; 1 fp32
    // as fp16 hi + lo, two MMAs per k-step; 2 fp32 as hi and lo in adjacent
    // MMA columns, one MMA per k-step (M <= 4)
    int xmode = 0;
    size_t smem = 0;
    size_t xf_bytes = 0, xs_bytes = 0, ws_bytes = 0;
    int split_counters = 0;
};

// allow_xstream: 0 when the kernel builds the fragments itself (fused fill),
// which needs them resident.
int plan_gemv(const DevMatrix &w, int M, int mode, bool xsplit, GemvPlan *plan, bool allow_xstream = true);

// Fragment fills write the row unscale factors xe[M] (2^-e of the row's
// power-of-two scaling) beside the block sums.
cudaError_t launch_xfill_f16(const XSrc &s, int M, int K, int Kp, int e_cols, bool xsplit, int bits, void *xf,
                             float *xs, float *xe, cudaStream_t st, const FillExchange *ex = nullptr);
// Whether launch_xfill_f16 can fuse an exchange for rows of K (Kp padded)
// columns: every CTA's columns fit its threads' register cache.
bool xfill_exchange_fits(int M, int Kp);
cudaError_t launch_xmaterialize(const XSrc &s, int M, int K, int Kp, float *out, cudaStream_t st);

// x-fragment preparation (fp activations -> fp16 fragments + block sums).
cudaError_t launch_xprep_f16(const void *x, int x_dtype, int M, int K, int Kp, int e_cols, bool xsplit, int bits,
                             void *xf, float *xs, float *xe, cudaStream_t st);
// int8 activations -> int8 fragments.
cudaError_t launch_xprep_s8(const int8_t *xq, int M, int K, int Kp, void *xf, cudaStream_t st);
// fp32 activations -> per-row dynamic int8 quantization (+ fragments).
cudaError_t launch_act_quant_s8(const float *x, int M, int K, int Kp, int8_t *q, float *scales, void *xf,
                                cudaStream_t st);

cudaError_t launch_gemv(const DevMatrix &w0, const DevMatrix *w1, const GemvPlan &plan, const GemvParams &p,
                        cudaStream_t st);

// Prefill dequant-GEMM (prefill.cu).
size_t prefill_xt_bytes(int M, int K);
bool prefill_supported(const DevMatrix &w);
cudaError_t launch_prefill(const DevMatrix &w, const void *x, int x_dtype, int M, void *xt, float *y, int ldy,
                           int accumulate, int *err, cudaStream_t st);

// Repack row-major codes of `src_bits` bits each (LSB first inside a byte;
// src_bits = 8 for one byte per code) into the code area of the strip layout
// of `m`, XOR-ing each code with `xorv` (F16 layout only).
cudaError_t launch_repack_codes(const uint8_t *src, size_t row_stride, int src_bits, uint32_t xorv,
                                const DevMatrix &m, cudaStream_t st);
// Read-back of a matrix in strip layout: row-major codes packed LSB first
// (row_bytes per row, the stored XOR undone) and its group metadata (fp16
// scales / zeros [N][n_groups], or the fp32 per-row scale of kMetaF32).
cudaError_t launch_unpack(const DevMatrix &m, uint32_t xorv, size_t row_bytes, uint8_t *codes, __half *s, __half *z,
                          float *fs, cudaStream_t st);
// Grouped quantization of fp32 weights [N][K] (one code byte per weight).
cudaError_t launch_quant_group(const float *w, int N, int K, int group, int bits, int symmetric, uint8_t *codes,
                               __half *scales, __half *zeros, cudaStream_t st);
// Scales [N][n_groups] (fp16, with fp16 zeros) or per-row fp32 scale/offset
// -> the metadata area of every block of `m`.
cudaError_t launch_meta_repack(const __half *s, const __half *z, const float *fs, const float *fo,
                               float zc_for_f32, const DevMatrix &m, cudaStream_t st);

}  // namespace chpe
