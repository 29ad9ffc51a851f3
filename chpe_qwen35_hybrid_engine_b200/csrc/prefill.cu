// prefill.cu -- dequant-GEMM for prefill (M >= 64 activation rows) on the
// 5th-generation tensor cores: y[M, N] = x[M, K] . dequant(W)[N, K]^T.
//
// One CTA computes a tile of 256 weight rows x 256 tokens of y over all of K
// in steps of 64 columns (a "k-block"), as two 128 x 256 MMA accumulators
// (all 512 TMEM columns) that share each activation tile.  The weights are the
// MMA's M side, so each dequantized weight tile serves 256 tokens and the
// accumulators' TMEM lanes are weight rows (the epilogue's stores are 128-byte
// rows of y); sharing the activation tile between two weight halves halves
// the operand bytes each MMA cycle needs, which is what lets a 3-stage ring
// cover the L2 / HBM latency:
//   * warp 0, one lane: three copies per k-block on the TMA engine (mbarrier
//     transaction counts) into a 3-stage input ring: the activation tile
//     (1-D bulk copy of 256 x 64 fp16) and, through two 3-D tensor maps over
//     the decode path's strip layout (words of a block x blocks x strips; one
//     copy of the weights in HBM), the 1 or 2 chunks of codes and the group
//     metadata that cover the k-block for the tile's 16 strips (strips past
//     the matrix read as zeros).
//   * warps 4..19: warp 4 + i dequantizes strip i (16 weight rows x 64) into
//     fp16 in shared memory, in the UMMA canonical K-major layout with the
//     128-byte swizzle (two 128-row tiles stacked), into a 2-stage ring.  A code becomes an exact fp16
//     integer with one byte-permute / LOP3 against the bit pattern of 1024
//     (0x6400), one HSUB2 removes 1024 + 128 (signed int8) or 1024 + zero, and
//     one HMUL2 applies the group scale: w = fp16(q * s), a single rounding.
//     The strip layout keeps each lane's codes in MMA-fragment register order,
//     which is exactly what stmatrix takes: one stmatrix.x4 writes a 16 x 16
//     block of the tile.
//   * warp 1, one lane: tcgen05.mma.cta_group::1.kind::f16 (A = weights,
//     B = activations, both fp16 from shared memory, fp32 accumulators of
//     128 x 256 in tensor memory), 2 x 4 instructions of K = 16 per k-block;
//     tcgen05.commit frees the stages once the MMAs that read them finish.
//   * warps 4..19 again, after the last k-block: tcgen05.ld the accumulators
//     (warp 4 + 4c + q reads TMEM lanes 32q..32q+31 = weight rows of half
//     c & 1, token columns 128 (c >> 1) .. +127) and store fp32 into y.
// Activations are converted once per call into fp16 tiles of 256 x 64 already
// in the swizzled layout (chpe_prefill_xprep_kernel), so each k-block's B operand
// is one contiguous 32 KB copy.  Every wait is bounded: on a timeout the
// kernel records an error code, stops issuing, waits (bounded) for the work it
// issued, frees its tensor memory and returns.
#include <cuda.h>  // CUtensorMap and its enums (the encoder is fetched at run time)

#include <algorithm>

#include "../../include/chpe_b200.h"
#include "common.cuh"
#include "internal.h"
#include "xsrc.cuh"

namespace chpe {
namespace {

constexpr int kPM = 128;          // weight rows per MMA (UMMA M, cta_group::1)
constexpr int kPHalves = 2;       // MMA accumulators (weight halves) per CTA
constexpr int kPN = 256;          // tokens per tile (UMMA N)
constexpr int kPK = 64;           // columns per k-block (one 128-byte swizzle atom of fp16)
constexpr int kInStages = 3;      // activation + packed-weight ring
constexpr int kWStages = 2;       // dequantized weight ring
constexpr int kPThreads = 640;    // 20 warps
constexpr int kDeqWarp0 = 4;      // first dequant / epilogue warp
constexpr int kDeqWarps = 16;
constexpr int kStripsPerTile = kPHalves * kPM / kStripRows;  // 16
constexpr uint32_t kWHalfBytes = kPM * kPK * 2;              // 16 KB of fp16 weights per MMA
constexpr uint32_t kWTileBytes = kPHalves * kWHalfBytes;     // 32 KB
constexpr uint32_t kXTileBytes = kPN * kPK * 2;              // 32 KB of fp16 activations
constexpr uint32_t kTmemCols = kPHalves * kPN;               // 512: the whole tensor memory
static_assert(kDeqWarps == kStripsPerTile, "one dequant warp per strip");

enum PrefillErr : int { kPErrInFull = 21, kPErrInEmpty = 22, kPErrBFull = 23, kPErrBEmpty = 24, kPErrAcc = 25 };

// Byte offset of element (row, k) (k < 64) inside a K-major, 128-byte
// swizzled fp16 tile: 8-row atoms of 1024 B, 16-byte chunk index XOR row.
__host__ __device__ __forceinline__ uint32_t swz_off(int row, int k) {
    return (uint32_t)((row >> 3) * 1024 + (row & 7) * 128 + ((((k >> 3) ^ (row & 7)) & 7) << 4) + (k & 7) * 2);
}

// UMMA shared-memory descriptor of a K-major, 128-byte swizzled operand
// (sm_100 format: start >> 4 in [0,14), LBO >> 4 in [16,30), SBO >> 4 in
// [32,46), version 1 at bit 46, layout type 2 = SWIZZLE_128B in [61,64)).
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t smem_addr) {
    uint64_t d = (uint64_t)((smem_addr >> 4) & 0x3FFFu);
    d |= (uint64_t)1u << 16;     // leading byte offset: 16 B (unused by the swizzled K-major layout)
    d |= (uint64_t)64u << 32;    // stride byte offset: 1024 B between 8-row atoms
    d |= (uint64_t)1u << 46;     // descriptor version for sm_100
    d |= (uint64_t)2u << 61;     // SWIZZLE_128B
    return d;
}

// Instruction descriptor of kind::f16: fp32 accumulator, fp16 A and B, both
// K-major, M = 128 (weight rows), N = 256 (tokens).
constexpr uint32_t kIdesc = (1u << 4) | ((uint32_t)(kPN >> 3) << 17) | ((uint32_t)(kPM >> 4) << 24);

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(kIdesc), "r"(accumulate)
        : "memory");
}

// Arrive on `bar` once every tcgen05.mma issued so far by this thread is done.
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld16(uint32_t addr, uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(addr));
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Tiled copy of a box of a 3-D tensor map into this CTA's shared memory.
__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map, int x, int y, int z, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
        "[%5];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
        : "memory");
}

// Four 8 x 8 fp16 matrices from MMA-fragment registers to shared memory: lane
// i gives the address of row i % 8 of matrix i / 8; register j of every lane
// holds (row lane / 4, columns 2 (lane % 4), +1) of matrix j.
__device__ __forceinline__ void stmatrix_x4(uint32_t addr, uint32_t r0, uint32_t r1, uint32_t r2, uint32_t r3) {
    asm volatile("stmatrix.sync.aligned.m8n8.x4.shared.b16 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(r0), "r"(r1),
                 "r"(r2), "r"(r3)
                 : "memory");
}

__device__ __forceinline__ uint32_t h2_bits(__half2 h) { return *reinterpret_cast<uint32_t *>(&h); }
__device__ __forceinline__ __half2 bits_h2(uint32_t u) { return *reinterpret_cast<__half2 *>(&u); }

struct PrefillParams {
    const uint8_t *codes;  // strip layout
    const uint16_t *xt;    // activation tiles [token_tile][k_block][256 x 64 swizzled fp16]
    const float2 *rs;      // per token (2^e, 2^-e): the row scaling applied before the fp16 conversion
    float *y;
    int ldy, M, N, K;
    int n_strips, n_blocks, block_bytes, bits, meta_kind, group, span;
    int n_kb;              // k-blocks (ceil(K / 64))
    int n_tt;              // token tiles (256 tokens each)
    float zc;              // constant zero-point (meta S16 with zero)
    int accumulate;
    int *err;
};

// Packed bytes of one strip for one k-block: codes then metadata.
struct KbSlice {
    uint32_t code_off, code_bytes, meta_off, meta_bytes;
    int g_first, g_per;    // first group of the k-block inside the block's metadata; columns per group (<= 64: group)
};

__host__ __device__ inline KbSlice kb_slice(const PrefillParams &p, int kb) {
    KbSlice s;
    const int k0 = kb * kPK;
    const int kin = k0 % p.span;            // column inside the block
    const int kc = 256 / p.bits;            // columns per chunk
    s.code_off = (uint32_t)(kin / kc) * kChunkBytes;
    s.code_bytes = (uint32_t)(kPK / kc > 0 ? kPK / kc : 1) * kChunkBytes;  // 8-bit: 2 chunks, 4-bit: 1
    const int mb = meta_bytes(p.meta_kind);
    const int gpb_cols = p.group <= p.span ? p.group : p.span;  // columns per stored group
    s.g_first = kin / gpb_cols;
    const int ng = gpb_cols >= kPK ? 1 : kPK / gpb_cols;
    s.g_per = gpb_cols;
    s.meta_off = (uint32_t)kBlockCodeBytes + (uint32_t)(s.g_first * 16 * mb);
    s.meta_bytes = (uint32_t)(ng * 16 * mb);
    return s;
}

struct PSmem {
    uint32_t in_full, in_empty, w_full, w_empty, acc, tmem_slot, in_ring, in_stage, w_ring, total;
};

// Input stage: [activation tile 32 KB][codes: 8 strips x code_bytes][metadata: 8 strips x meta_bytes].
__host__ __device__ inline PSmem psmem(uint32_t code_bytes, uint32_t meta_bytes) {
    PSmem L;
    L.in_full = 0;
    L.in_empty = L.in_full + 8 * kInStages;
    L.w_full = L.in_empty + 8 * kInStages;
    L.w_empty = L.w_full + 8 * kWStages;
    L.acc = L.w_empty + 8 * kWStages;
    L.tmem_slot = L.acc + 8;
    L.in_stage = (kXTileBytes + kStripsPerTile * (code_bytes + meta_bytes) + 1023u) & ~1023u;
    L.in_ring = 1024;  // stages 1024-aligned (the swizzle is a function of the address)
    L.w_ring = L.in_ring + kInStages * L.in_stage;
    L.total = L.w_ring + kWStages * kWTileBytes;
    return L;
}

template <int BITS, int META>
__global__ void __launch_bounds__(kPThreads, 1)
    chpe_prefill_gemm_kernel(const PrefillParams p, const __grid_constant__ CUtensorMap tm_codes,
                        const __grid_constant__ CUtensorMap tm_meta) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // the swizzle is a function of the address: align the working area to 1024 B
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tt = blockIdx.x % p.n_tt, wt = blockIdx.x / p.n_tt;  // tiles sharing weights run together
    const int tok0 = tt * kPN, strip0 = wt * kStripsPerTile;

    const KbSlice s0 = kb_slice(p, 0);  // sizes are the same for every k-block
    const PSmem L = psmem(s0.code_bytes, s0.meta_bytes);
    uint64_t *in_full = reinterpret_cast<uint64_t *>(smem + L.in_full);
    uint64_t *in_empty = reinterpret_cast<uint64_t *>(smem + L.in_empty);
    uint64_t *w_full = reinterpret_cast<uint64_t *>(smem + L.w_full);
    uint64_t *w_empty = reinterpret_cast<uint64_t *>(smem + L.w_empty);
    uint64_t *acc_bar = reinterpret_cast<uint64_t *>(smem + L.acc);
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + L.tmem_slot);

    if (threadIdx.x == 0) {
        for (int s = 0; s < kInStages; ++s) {
            mbar_init(&in_full[s], 1);
            mbar_init(&in_empty[s], 1 + kDeqWarps);  // MMA commit + every dequant warp
        }
        for (int s = 0; s < kWStages; ++s) {
            mbar_init(&w_full[s], kDeqWarps);
            mbar_init(&w_empty[s], 1);
        }
        mbar_init(acc_bar, 1);
        fence_barrier_init();
        grid_dependents_launch();
    }
    if (warp == 1) {  // the whole warp allocates the accumulator's tensor memory
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_d = *tmem_slot;
    const int n_kb = p.n_kb;

    if (warp == 0) {
        // ---------------- producer ----------------
        if (lane == 0) {
            int kb = 0;
            bool waited = false;
            for (; kb < n_kb; ++kb) {
                const int s = kb % kInStages, use = kb / kInStages;
                if (use > 0 && !mbar_wait_bounded(&in_empty[s], (use - 1) & 1)) {
                    atomicExch(p.err, kPErrInEmpty);
                    break;
                }
                uint8_t *stage = smem + L.in_ring + s * L.in_stage;
                const KbSlice ks = kb_slice(p, kb);
                const int blk = (kb * kPK) / p.span;
                // full boxes land even for strips past the matrix (zero-filled)
                mbar_arrive_expect_tx(&in_full[s], kXTileBytes + kStripsPerTile * (ks.code_bytes + ks.meta_bytes));
                tma_load_3d(stage + kXTileBytes, &tm_codes, (int)(ks.code_off / 4), blk, strip0, &in_full[s]);
                tma_load_3d(stage + kXTileBytes + kStripsPerTile * ks.code_bytes, &tm_meta, (int)(ks.meta_off / 4),
                            blk, strip0, &in_full[s]);
                if (!waited) {  // the activation tiles come from the previous kernel
                    grid_dependency_wait();
                    waited = true;
                }
                bulk_g2s(stage, p.xt + ((size_t)tt * n_kb + kb) * (kPN * kPK), kXTileBytes, &in_full[s]);
            }
            // every issued copy has landed before the CTA may leave
            for (int s = 0; s < kInStages && s < kb; ++s) {
                const int last = s + ((kb - 1 - s) / kInStages) * kInStages;
                if (!mbar_wait_bounded(&in_full[s], (last / kInStages) & 1)) atomicExch(p.err, kPErrInFull);
            }
        }
    } else if (warp == 1) {
        // ---------------- MMA issue ----------------
        if (lane == 0) {
            for (int kb = 0; kb < n_kb; ++kb) {
                const int s = kb % kInStages, ws = kb % kWStages;
                if (!mbar_wait_bounded(&in_full[s], (kb / kInStages) & 1)) {
                    atomicExch(p.err, kPErrInFull);
                    break;
                }
                if (!mbar_wait_bounded(&w_full[ws], (kb / kWStages) & 1)) {
                    atomicExch(p.err, kPErrBFull);
                    break;
                }
                tc_fence_after();
                const uint32_t x_base = smem_u32(smem + L.in_ring + s * L.in_stage);
                const uint32_t w_base = smem_u32(smem + L.w_ring + ws * kWTileBytes);
#pragma unroll
                for (int kk = 0; kk < kPK / 16; ++kk)
#pragma unroll
                    for (int a = 0; a < kPHalves; ++a)
                        umma_f16(tmem_d + (uint32_t)(a * kPN), umma_desc_sw128(w_base + a * kWHalfBytes + kk * 32),
                                 umma_desc_sw128(x_base + kk * 32), (kb > 0 || kk > 0) ? 1u : 0u);
                umma_commit(&in_empty[s]);  // activation stage free once these MMAs are done
                umma_commit(&w_empty[ws]);  // and the dequantized weight stage
            }
            umma_commit(acc_bar);  // the accumulator is complete (or this CTA gave up)
            // the MMAs issued read shared memory: they finish before the CTA leaves
            if (!mbar_wait_bounded(acc_bar, 0)) atomicExch(p.err, kPErrAcc);
        }
    } else if (warp >= kDeqWarp0) {
        // ---------------- dequant, then epilogue ----------------
        const int dw = warp - kDeqWarp0;  // 0..15: strip dw of the tile, weight rows 16dw..16dw+15
        const int g = lane >> 2;
        // stmatrix address of this lane inside a 16 x 16 block: row (lane % 8) + 8 ((lane / 8) & 1) of the
        // strip, columns 8 (lane / 16) .. +7 of the k-step
        const int st_row = 16 * dw + (lane & 7) + 8 * ((lane >> 3) & 1);
        const int st_col = 8 * (lane >> 4);
        bool ok = true;
        for (int kb = 0; kb < n_kb; ++kb) {
            const int s = kb % kInStages, ws = kb % kWStages;
            if (!__all_sync(0xffffffffu, mbar_wait_bounded(&in_full[s], (kb / kInStages) & 1))) {
                if (lane == 0) atomicExch(p.err, kPErrInFull);
                ok = false;
                break;
            }
            if (kb >= kWStages &&
                !__all_sync(0xffffffffu, mbar_wait_bounded(&w_empty[ws], ((kb / kWStages) - 1) & 1))) {
                if (lane == 0) atomicExch(p.err, kPErrBEmpty);
                ok = false;
                break;
            }
            const uint8_t *stage = smem + L.in_ring + s * L.in_stage;
            const uint8_t *sp = stage + kXTileBytes + dw * s0.code_bytes;                                // codes
            const uint8_t *mp = stage + kXTileBytes + kStripsPerTile * s0.code_bytes + dw * s0.meta_bytes;  // metadata
            const uint32_t wt_base = smem_u32(smem + L.w_ring + ws * kWTileBytes);
            if constexpr (BITS == 8) {
                // two chunks of 32 columns (2 k-steps each); group 32 = one scale per chunk and row
#pragma unroll
                for (int h = 0; h < 2; ++h) {
                    const uint4 wv = *reinterpret_cast<const uint4 *>(sp + h * kChunkBytes + lane * 16);
                    const uint32_t w4[4] = {wv.x, wv.y, wv.z, wv.w};
                    // scales of rows g and g + 8, stored side by side
                    const __half2 sp2 = *reinterpret_cast<const __half2 *>(mp + ((h * 32) / s0.g_per) * 32 + 4 * g);
                    const __half2 s_lo = __low2half2(sp2), s_hi = __high2half2(sp2);
                    const __half2 off = __float2half2_rn(1152.0f);  // 1024 + 128: u = q + 128
                    uint32_t a[2][4];
#pragma unroll
                    for (int r = 0; r < 4; ++r) {
                        const __half2 sc = (r & 1) ? s_hi : s_lo;
                        a[0][r] = h2_bits(__hmul2(__hsub2(bits_h2(__byte_perm(w4[r], 0x64646464u, 0x4140)), off), sc));
                        a[1][r] = h2_bits(__hmul2(__hsub2(bits_h2(__byte_perm(w4[r], 0x64646464u, 0x4342)), off), sc));
                    }
#pragma unroll
                    for (int j = 0; j < 2; ++j)
                        stmatrix_x4(wt_base + swz_off(st_row, 32 * h + 16 * j + st_col), a[j][0], a[j][1], a[j][2],
                                    a[j][3]);
                }
            } else {
                // one chunk of 64 columns (4 k-steps); nibble j -> k-step j, nibble j+4 -> its next column
                const uint4 wv = *reinterpret_cast<const uint4 *>(sp + lane * 16);
                const uint32_t w4[4] = {wv.x, wv.y, wv.z, wv.w};
                __half2 s2[2], z2[2];
                if constexpr (META == kMetaSZ16) {
                    // (scale, zero) of rows g and g + 8, stored side by side
                    const uint2 v = *reinterpret_cast<const uint2 *>(mp + 8 * g);
                    const __half2 a0 = bits_h2(v.x), a1 = bits_h2(v.y);
                    s2[0] = __low2half2(a0);
                    s2[1] = __low2half2(a1);
                    z2[0] = __hadd2(__high2half2(a0), __float2half2_rn(1024.0f));  // 1024 + z (exact: z < 1024)
                    z2[1] = __hadd2(__high2half2(a1), __float2half2_rn(1024.0f));
                } else {
                    const __half2 sp2 = *reinterpret_cast<const __half2 *>(mp + 4 * g);
                    s2[0] = __low2half2(sp2);
                    s2[1] = __high2half2(sp2);
                    z2[0] = z2[1] = __float2half2_rn(1024.0f + p.zc);
                }
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    uint32_t a[4];
#pragma unroll
                    for (int r = 0; r < 4; ++r) {
                        const uint32_t e = ((w4[r] >> (4 * j)) & 0x000F000Fu) | 0x64006400u;  // (1024+c_a, 1024+c_b)
                        a[r] = h2_bits(__hmul2(__hsub2(bits_h2(e), z2[r & 1]), s2[r & 1]));
                    }
                    stmatrix_x4(wt_base + swz_off(st_row, 16 * j + st_col), a[0], a[1], a[2], a[3]);
                }
            }
            fence_async_smem();  // the generic-proxy stores become visible to the tensor cores
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&w_full[ws]);
                mbar_arrive(&in_empty[s]);
            }
        }
        // ---------------- epilogue ----------------
        if (ok && __all_sync(0xffffffffu, mbar_wait_bounded(acc_bar, 0))) {
            tc_fence_after();
            grid_dependency_wait();  // y may still be read by the previous kernel
            const int q = dw & 3;                   // TMEM lanes 32q..32q+31: weight rows of half `a`
            const int a = (dw >> 2) & 1;            // accumulator (weight half)
            const int c0 = (dw >> 3) * 128;         // token columns 0..127 or 128..255
            const int n = strip0 * kStripRows + a * kPM + 32 * q + lane;
#pragma unroll 1
            for (int cc = 0; cc < 128; cc += 16) {
                uint32_t v[16];
                tmem_ld16(tmem_d + ((uint32_t)(32 * q) << 16) + (uint32_t)(a * kPN + c0 + cc), v);
                tmem_ld_wait();
                if (n < p.N) {
#pragma unroll
                    for (int e = 0; e < 16; ++e) {
                        const int m = tok0 + c0 + cc + e;
                        if (m < p.M) {
                            float *yp = p.y + (size_t)m * p.ldy + n;
                            const float val = __uint_as_float(v[e]) * p.rs[m].y;  // undo the row scaling
                            *yp = p.accumulate ? *yp + val : val;
                        }
                    }
                }
            }
        } else if (lane == 0 && ok) {
            atomicExch(p.err, kPErrAcc);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_d), "r"(kTmemCols) : "memory");
    }
}

// Activations [M][K] (fp32 / bf16 / fp16) -> fp16 tiles [token_tile][k_block]
// of 256 x 64, K-major with the 128-byte swizzle; zero outside [M, K).  One
// thread per 8 consecutive columns (one 16-byte chunk of a tile row), read
// with vector loads where the row allows.
__device__ __forceinline__ float x_at(const void *x, int dt, size_t i) {
    return dt == CHPE_X_F32 ? static_cast<const float *>(x)[i]
           : dt == CHPE_X_BF16 ? __bfloat162float(static_cast<const __nv_bfloat16 *>(x)[i])
                               : __half2float(static_cast<const __half *>(x)[i]);
}

// Row scaling of the prefill activations: each token row's max |x| gives
// (2^e, 2^-e) with max |x| * 2^e in [2^14, 2^15) (row_scale_exp), so the
// fp16 tiles hold every row whatever its magnitude;
// the epilogue multiplies the row's sums by 2^-e (powers of two are exact).
// One warp per row (8 rows per CTA); rows whose start is 16-byte aligned and
// whose length is a whole number of 16-byte vectors are read 16 bytes per
// lane and load (all of a lane's loads in flight), the rest element-wise.
// max |x| does not depend on the order, so both give the same scale.
__device__ __forceinline__ float absmax16(uint32_t w, int dt) {
    float a, b;
    if (dt == CHPE_X_BF16) {
        a = __uint_as_float(w << 16);
        b = __uint_as_float(w & 0xffff0000u);
    } else {
        a = __half2float(__ushort_as_half((unsigned short)(w & 0xffffu)));
        b = __half2float(__ushort_as_half((unsigned short)(w >> 16)));
    }
    return fmaxf(fabsf(a), fabsf(b));
}

__global__ void __launch_bounds__(256) chpe_prefill_rowscale_kernel(const void *__restrict__ x, int dt, int M, int K,
                                                                   float2 *__restrict__ rs) {
    pdl_begin();
    const int lane = threadIdx.x & 31;
    const int m = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (m >= M) return;
    const size_t esz = dt == CHPE_X_F32 ? 4 : 2;
    const char *row = static_cast<const char *>(x) + (size_t)m * K * esz;
    const size_t bytes = (size_t)K * esz;
    float am = 0.0f;
    if ((reinterpret_cast<uintptr_t>(row) & 15) == 0 && (bytes & 15) == 0) {
        const uint4 *v = reinterpret_cast<const uint4 *>(row);
        const int nv = (int)(bytes / 16);
        for (int i = lane; i < nv; i += 32) {
            const uint4 q = __ldg(v + i);
            if (dt == CHPE_X_F32) {
                am = fmaxf(am, fmaxf(fmaxf(fabsf(__uint_as_float(q.x)), fabsf(__uint_as_float(q.y))),
                                     fmaxf(fabsf(__uint_as_float(q.z)), fabsf(__uint_as_float(q.w)))));
            } else {
                am = fmaxf(am, fmaxf(fmaxf(absmax16(q.x, dt), absmax16(q.y, dt)),
                                     fmaxf(absmax16(q.z, dt), absmax16(q.w, dt))));
            }
        }
    } else {
        for (int k = lane; k < K; k += 32) am = fmaxf(am, fabsf(x_at(x, dt, (size_t)m * K + k)));
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, off));
    if (lane == 0) {
        const int e = row_scale_exp(am);
        rs[m] = make_float2(pow2_of(e), pow2_of(-e));
    }
}

__global__ void chpe_prefill_xprep_kernel(const void *__restrict__ x, int dt, int M, int K, int n_tt, int n_kb,
                                          const float2 *__restrict__ rs, uint16_t *__restrict__ xt) {
    pdl_begin();
    const size_t total = (size_t)n_tt * kPN * n_kb * (kPK / 8);
    const bool vec = (K % 8) == 0 && (reinterpret_cast<uintptr_t>(x) % 16) == 0;
    for (size_t idx = (size_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
         idx += (size_t)gridDim.x * blockDim.x) {
        const int ch = (int)(idx % (kPK / 8));
        const size_t rest = idx / (kPK / 8);
        const int kb = (int)(rest % n_kb);
        const int m = (int)(rest / n_kb);
        const int k0 = kb * kPK + ch * 8;
        uint4 out = make_uint4(0u, 0u, 0u, 0u);
        if (m < M && k0 < K) {
            const size_t base = (size_t)m * K + k0;
            const float sc = rs[m].x;
            float f[8];
            if (vec && dt == CHPE_X_F16) {
                const uint4 v = *reinterpret_cast<const uint4 *>(static_cast<const __half *>(x) + base);
                const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float2 t = __half22float2(bits_h2(w[e]));
                    f[2 * e] = t.x;
                    f[2 * e + 1] = t.y;
                }
            } else if (vec && dt == CHPE_X_BF16) {
                const uint4 v = *reinterpret_cast<const uint4 *>(static_cast<const __nv_bfloat16 *>(x) + base);
                const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float2 t = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&w[e]));
                    f[2 * e] = t.x;
                    f[2 * e + 1] = t.y;
                }
            } else if (vec && dt == CHPE_X_F32) {
                const float4 a = *reinterpret_cast<const float4 *>(static_cast<const float *>(x) + base);
                const float4 b = *reinterpret_cast<const float4 *>(static_cast<const float *>(x) + base + 4);
                f[0] = a.x, f[1] = a.y, f[2] = a.z, f[3] = a.w, f[4] = b.x, f[5] = b.y, f[6] = b.z, f[7] = b.w;
            } else {
#pragma unroll
                for (int e = 0; e < 8; ++e) f[e] = k0 + e < K ? x_at(x, dt, base + e) : 0.0f;
            }
            uint32_t h[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) h[e] = h2_bits(__floats2half2_rn(f[2 * e] * sc, f[2 * e + 1] * sc));
            out = make_uint4(h[0], h[1], h[2], h[3]);
        }
        const int tt = m / kPN, r = m % kPN;
        uint8_t *tile = reinterpret_cast<uint8_t *>(xt) + ((size_t)tt * n_kb + kb) * kXTileBytes;
        *reinterpret_cast<uint4 *>(tile + swz_off(r, ch * 8)) = out;
    }
}

using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                   const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled() {
    static EncodeTiledFn fn = nullptr;
    if (!fn) {
        void *ptr = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(ptr);
        else
            cudaGetLastError();
    }
    return fn;
}

// The strip layout as a 3-D tensor of 32-bit words: (word of a block) x
// blocks x strips; the box is one word range of one block of 16 strips.
bool make_strip_map(CUtensorMap *map, const PrefillParams &p, uint32_t box_bytes) {
    EncodeTiledFn fn = encode_tiled();
    if (!fn) return false;
    const cuuint64_t dims[3] = {(cuuint64_t)(p.block_bytes / 4), (cuuint64_t)p.n_blocks, (cuuint64_t)p.n_strips};
    const cuuint64_t strides[2] = {(cuuint64_t)p.block_bytes, (cuuint64_t)p.block_bytes * (cuuint64_t)p.n_blocks};
    const cuuint32_t box[3] = {box_bytes / 4, 1, (cuuint32_t)kStripsPerTile};
    const cuuint32_t estr[3] = {1, 1, 1};
    return fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT32, 3, const_cast<uint8_t *>(p.codes), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int BITS, int META>
cudaError_t launch_prefill_t(const PrefillParams &p, size_t smem, cudaStream_t st) {
    auto kern = chpe_prefill_gemm_kernel<BITS, META>;
    static KernelDeviceState kstate;  // the shared-memory limit is set once per device
    cudaError_t pe = kernel_prepare(kstate, kern, kPThreads, smem, smem, nullptr);
    if (pe != cudaSuccess) return pe;
    const KbSlice s0 = kb_slice(p, 0);
    CUtensorMap tm_codes, tm_meta;
    if (!make_strip_map(&tm_codes, p, s0.code_bytes) || !make_strip_map(&tm_meta, p, s0.meta_bytes))
        return cudaErrorInvalidValue;
    const int n_wt = (p.n_strips + kStripsPerTile - 1) / kStripsPerTile;
    return launch_pdl(kern, dim3((unsigned)(p.n_tt * n_wt)), dim3(kPThreads), smem, st, p, tm_codes, tm_meta);
}

}  // namespace

// Scratch bytes for the activation tiles of an M x K prefill, then the
// per-token row scales (float2 per token of the padded token tiles).
size_t prefill_tiles_bytes(int M, int K) {
    const size_t n_tt = (size_t)(M + kPN - 1) / kPN, n_kb = (size_t)(K + kPK - 1) / kPK;
    return n_tt * n_kb * kXTileBytes;
}
size_t prefill_xt_bytes(int M, int K) {
    const size_t n_tt = (size_t)(M + kPN - 1) / kPN;
    return prefill_tiles_bytes(M, K) + n_tt * kPN * sizeof(float2);
}

// Whether the prefill kernel handles this weight format.
bool prefill_supported(const DevMatrix &w) {
    if (w.layout != kLayoutF16) return false;
    if (w.bits == 8) return w.meta_kind == kMetaS16 && w.group == 32;
    if (w.bits == 4) return (w.meta_kind == kMetaSZ16 || w.meta_kind == kMetaS16) && w.group >= 64 &&
                            (w.group % 64) == 0;
    return false;
}

cudaError_t launch_prefill(const DevMatrix &w, const void *x, int x_dtype, int M, void *xt, float *y, int ldy,
                           int accumulate, int *err, cudaStream_t st) {
    PrefillParams p;
    p.codes = w.codes;
    p.xt = static_cast<const uint16_t *>(xt);
    float2 *rs = reinterpret_cast<float2 *>(static_cast<uint8_t *>(xt) + prefill_tiles_bytes(M, w.K));
    p.rs = rs;
    p.y = y;
    p.ldy = ldy;
    p.M = M;
    p.N = w.N;
    p.K = w.K;
    p.n_strips = w.n_strips;
    p.n_blocks = w.n_blocks;
    p.block_bytes = w.block_bytes;
    p.bits = w.bits;
    p.meta_kind = w.meta_kind;
    p.group = w.group;
    p.span = w.span;
    p.n_kb = (w.K + kPK - 1) / kPK;
    p.n_tt = (M + kPN - 1) / kPN;
    p.zc = w.zc;
    p.accumulate = accumulate;
    p.err = err;
    const size_t total = (size_t)p.n_tt * kPN * p.n_kb * (kPK / 8);
    cudaError_t e =
        launch_pdl(chpe_prefill_rowscale_kernel, dim3((unsigned)((M + 7) / 8)), dim3(256), 0, st, x, x_dtype, M, w.K, rs);
    if (e != cudaSuccess) return e;
    e = launch_pdl(chpe_prefill_xprep_kernel, dim3((unsigned)std::min<size_t>((total + 255) / 256, 148 * 16)),
                   dim3(256), 0, st, x, x_dtype, M, w.K, p.n_tt, p.n_kb, static_cast<const float2 *>(rs),
                   static_cast<uint16_t *>(xt));
    if (e != cudaSuccess) return e;
    const KbSlice s0 = kb_slice(p, 0);
    const size_t smem = psmem(s0.code_bytes, s0.meta_bytes).total + 1024;  // + alignment slack
    if (w.bits == 8) return launch_prefill_t<8, kMetaS16>(p, smem, st);
    if (w.meta_kind == kMetaSZ16) return launch_prefill_t<4, kMetaSZ16>(p, smem, st);
    return launch_prefill_t<4, kMetaS16>(p, smem, st);
}

}  // namespace chpe
