// layout.h -- device layout of quantized weight matrices ("strip layout") and
// of activation fragments, shared by host and device code.
//
// Strip layout.  A [N, K] matrix of `bits`-wide codes is cut into strips of 16
// rows.  Along K a strip is a run of blocks; a block is 8 chunks of codes
// (8 x 512 B = 4 KiB) followed by the metadata of the groups those chunks
// cover, so one 1-D bulk copy per strip and pipeline stage brings everything a
// warp needs.  One chunk is one warp-wide 128-bit load (32 lanes x 16 B) and
// covers KC = 256/bits columns; a block covers SPAN = 8*KC columns.  Lane
// l = 4*g + t holds, in its 16 bytes, the codes it feeds to the warp MMA as
// its A fragment (rows g and g+8 of the strip), so a lane never shuffles:
//   * F16 layout (m16n8k16, fp16 operands): register r (r = 0..3) of the lane
//     covers row g + 8*(r&1), columns c = 2t + 8*(r>>1) and c+1 of every
//     16-column k-step j.  4-bit: nibble j holds column 16j+c, nibble j+4
//     holds 16j+c+1.  2-bit: field j holds 16j+c, field j+8 holds 16j+c+1.
//     8-bit: bytes (2j, 2j+1) hold columns 16j+c, 16j+c+1 (j = 0, 1).
//   * S8 layout (m16n8k32, int8 operands): register r holds row g + 8*(r&1),
//     columns 4t + 16*(r>>1) + 0..3 of the 32-column k-step.
// Codes are stored unsigned in the F16 layout: signed int8 as q ^ 0x80, the
// 2-bit codebook {0:0,1:+1,2:-2,3:-1} as c ^ 2 (value = code - 2), offset-8
// nibbles as is.  The S8 layout keeps signed int8.
//
// Block metadata: [group-in-block][16 rows] entries of half (scale), half2
// (scale, zero) or float2 (scale, offset).  A block holds SPAN/group groups
// when group <= SPAN, else the single group it lies in (a per-row scale is
// repeated in every block).  K is padded to whole blocks with zero codes and
// zero metadata; activations are zero-padded, so padding contributes 0.
//
// Activation fragments (B operand): for each 16-column k-step s and activation
// row m < M, four uint2 (one per t): {x[16s+2t], x[16s+2t+1]}, {x[16s+2t+8],
// x[16s+2t+9]} as fp16 pairs; layout [kstep][M][4].  fp32 activations are
// carried as hi + lo fp16 pairs (two fragment arrays).  Sums of the fp16
// values over each E-column block, [eblock][8] fp32, let the epilogue apply the
// zero-point as  s*sum(c*x) - s*z*sum(x).  int8 activations use [kstep32][M][4]
// uint2 = {x[32s+4t..+3], x[32s+4t+16..+19]}.
#pragma once
#include <stdint.h>

#if defined(__CUDACC__)
#define CHPE_HD __host__ __device__
#else
#define CHPE_HD
#endif

namespace chpe {

constexpr int kStripRows = 16;
constexpr int kChunkBytes = 512;
constexpr int kChunksPerBlock = 8;
constexpr int kBlockCodeBytes = kChunksPerBlock * kChunkBytes;
constexpr int kMaxTokens = 8;  // activation rows per MMA n-tile

enum LayoutKind : int { kLayoutF16 = 0, kLayoutS8 = 1 };
enum MetaKind : int { kMetaNone = 0, kMetaS16 = 1, kMetaSZ16 = 2, kMetaF32 = 3 };

CHPE_HD inline constexpr int chunk_cols(int bits) { return 256 / bits; }
CHPE_HD inline constexpr int block_cols(int bits) { return kChunksPerBlock * chunk_cols(bits); }
CHPE_HD inline constexpr int meta_bytes(int kind) {
    return kind == kMetaS16 ? 2 : kind == kMetaSZ16 ? 4 : kind == kMetaF32 ? 8 : 0;
}
CHPE_HD inline constexpr int ceil_div(long a, long b) { return (int)((a + b - 1) / b); }

}  // namespace chpe
