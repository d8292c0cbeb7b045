// layout.cuh -- HBM tile layout of packed expert matrices.
//
// A matrix with K inputs and N outputs (both multiples of 128) is stored as blocks of
// 128 output channels x 128 inputs, ordered [n_tile][k_tile][slot], where `slot`
// interleaves gate (0) and up (1) for the fused gate/up matrix and is always 0 for a lone
// matrix.  One block is exactly what one pipeline stage of the grouped GEMM consumes, so
// a stage is a single contiguous bulk copy.
//
// Inside a block the weights are pre-arranged in tensor-core A-fragment order
// (mma m16n8k16, rows = output channels, cols = k): channel block cb (16 channels) x
// k chunk kc, 32 lanes x 16 bytes per (cb, kc).  A lane's 128-bit load therefore holds
// the fragments it feeds to the MMA with no shuffling.
//
//   AWQ int4 block (8512 B):  [0, 8192)     8 cb x 2 kc(64 k) x 32 lanes x 4 words
//                             [8192, 8448)  fp16 scale of each of the 128 channels
//                             [8448, 8512)  zero-point nibbles, channel c in byte c/2,
//                                           low nibble for even c
//     word j of a lane covers k-step j (16 k) of the chunk; nibble p of the word is
//     A-tile element (row g + 8*(p&1), col 2t + (p>>2) + 8*((p>>1)&1)), g = lane/4,
//     t = lane%4.  (w >> 4r) & 0x000F000F is then A register r as two 16-bit halves.
//   FP8 e4m3 block (16400 B): [0, 16384)    8 cb x 4 kc(32 k) x 32 lanes x 16 bytes
//                             [16384, 16388) fp32 block scale, 12 bytes padding
//     bytes [8j, 8j+8) of a lane cover k-step j; byte b is A-tile element
//     (row g + 8*((b>>1)&1), col 2t + 8*(b>>2) + (b&1)), i.e. byte pair r is A register r.
//   FP8 e4m3 channel-scaled block (16896 B): the FP8 codes as above, then at 16384 the fp32
//     scale of each of the 128 channels (for this 128-k group).
//   Signed int4 block (8704 B): the AWQ nibbles as above holding q = v + 8 (zero point 8 for
//     every channel), then at 8192 the fp32 scale of each of the 128 channels.
//
// Row layout (used by the tcgen05 kernel): the same block sizes, but each block holds one
// output channel per row (one tensor-memory lane of the A operand) and is split into two
// contiguous 64-k halves, so that one pipeline stage (64 k) is one contiguous copy:
//   AWQ int4: half h at [4096 h, 4096 h + 4096): 128 rows x 32 B; 16-byte chunk c (0..1) of
//             row r at r*32 + 16*(c ^ ((r >> 2) & 1)); word j (0..3) of a chunk covers
//             k = 64h + 32c + 8j .. +7 with nibble slot p holding k offset {0,2,4,6,1,3,5,7}[p],
//             so (w >> 4i) & 0x000F000F is the pair (2i, 2i+1).  Scales at 8192, zero-point
//             nibbles at 8448, per row, as above.
//   FP8:      half h at [8192 h, 8192 h + 8192): 128 rows x 64 B; chunk c (0..3) of row r at
//             r*64 + 16*(c ^ ((r >> 1) & 3)); byte b of a chunk is k = 64h + 16c + b.  Scale at
//             16384 (a fused gate/up block: gate scale at 16384, up scale at 16388; the scale
//             of row r is at 16384 + 4 (r & 1)).
//   The channel-scaled formats keep the codes of their base format and one fp32 scale per
//   row at the scale offset (row r of a fused gate/up block: the scale of its channel).
// The XOR swizzle makes the eight rows read by each quarter-warp hit eight distinct bank
// groups.  A lone matrix (down projection) uses blocks of 128 channels; the gate and up
// matrices are fused: block t holds gate channel 64t + i in row 2i and the up channel of the
// same index in row 2i + 1, so that one 128-row MMA tile yields both halves of SwiGLU and the
// two sums of a channel sit in adjacent tensor-memory lanes (one warp's lanes 2i, 2i + 1).
#pragma once

#include "common.cuh"

namespace ccut {

constexpr int kTileN = 128;  // output channels per block
constexpr int kTileK = 128;  // inputs per block (= AWQ group = FP8 block)
constexpr int kMaxExperts = 512;

enum { kLayoutRows = 0, kLayoutFrags = 1 };

// Byte offset, inside a row-layout AWQ block, of the 32-bit word holding element k of row r.
inline __host__ __device__ int rows_awq_word(int r, int k) {
  const int h = k >> 6, c = (k >> 5) & 1, j = (k >> 3) & 3;
  return h * 4096 + r * 32 + 16 * (c ^ ((r >> 2) & 1)) + 4 * j;
}
inline __host__ __device__ int rows_awq_slot(int k) {  // nibble slot inside the word
  const int kk = k & 7;
  return (kk & 1) ? 4 + (kk >> 1) : (kk >> 1);
}
inline __host__ __device__ int rows_fp8_byte(int r, int k) {
  const int h = k >> 6, c = (k >> 4) & 3;
  return h * 8192 + r * 64 + 16 * (c ^ ((r >> 1) & 3)) + (k & 15);
}
// Source channel of row r of row-layout block `nt` for matrix `slot` (-1: the row belongs to
// the other matrix of a fused gate/up block, whose rows interleave: row 2i is gate channel
// 64 nt + i, row 2i + 1 the up channel of the same index).
inline __host__ __device__ int rows_channel(int nt, int r, int nmat, int slot) {
  if (nmat == 1) return nt * 128 + r;
  return (r & 1) == slot ? nt * 64 + (r >> 1) : -1;
}
// Row-layout blocks along the channel axis of a matrix with N channels.
inline __host__ __device__ int rows_nblocks(int N, int nmat) { return nmat == 1 ? N / 128 : N / 64; }

// Scale kinds: fp16 per channel (AWQ), one fp32 per block (FP8 b128), fp32 per channel.
enum { kScaleF16Row = 0, kScaleF32Block = 1, kScaleF32Row = 2 };

struct BlkInt4 {                            // nibble codes (AWQ and signed int4)
  static constexpr bool kInt4 = true;
  static constexpr int kChunks = 2;         // k chunks of 64 per channel block
  static constexpr int kChunkK = 64;
  static constexpr int kStepsPerChunk = 4;  // 16-k MMA steps per chunk
  static constexpr int kAtomBytes = 8192;
  static constexpr int kScaleOff = 8192;
  static constexpr bool kBf16 = false;  // f16 operands ((q - z) is exact in f16)
};

struct BlkE4m3 {  // e4m3 codes
  static constexpr bool kInt4 = false;
  static constexpr int kChunks = 4;  // k chunks of 32
  static constexpr int kChunkK = 32;
  static constexpr int kStepsPerChunk = 2;
  static constexpr int kAtomBytes = 16384;
  static constexpr int kScaleOff = 16384;
  static constexpr int kZeroOff = 0;
  static constexpr bool kZeros = false;
  static constexpr bool kBf16 = false;  // f16 operands (e4m3 -> f16 is exact)
};

template <int FMT>
struct Blk;

template <>
struct Blk<CCUT_FMT_AWQ_INT4_G128> : BlkInt4 {
  static constexpr int kZeroOff = 8448;
  static constexpr bool kZeros = true;  // 4-bit zero point per channel
  static constexpr int kScale = kScaleF16Row;
  static constexpr int kBytes = 8512;
};

template <>
struct Blk<CCUT_FMT_INT4_SYM_G128> : BlkInt4 {
  static constexpr int kZeroOff = 0;
  static constexpr bool kZeros = false;  // zero point 8
  static constexpr int kScale = kScaleF32Row;
  static constexpr int kBytes = 8704;
};

template <>
struct Blk<CCUT_FMT_FP8_E4M3_B128> : BlkE4m3 {
  static constexpr int kScale = kScaleF32Block;
  static constexpr int kBytes = 16400;
};

template <>
struct Blk<CCUT_FMT_FP8_E4M3_CH> : BlkE4m3 {
  static constexpr int kScale = kScaleF32Row;
  static constexpr int kBytes = 16896;
};

inline __host__ __device__ size_t block_bytes(int fmt) {
  switch (fmt) {
    case CCUT_FMT_AWQ_INT4_G128: return Blk<CCUT_FMT_AWQ_INT4_G128>::kBytes;
    case CCUT_FMT_INT4_SYM_G128: return Blk<CCUT_FMT_INT4_SYM_G128>::kBytes;
    case CCUT_FMT_FP8_E4M3_CH: return Blk<CCUT_FMT_FP8_E4M3_CH>::kBytes;
    default: return Blk<CCUT_FMT_FP8_E4M3_B128>::kBytes;
  }
}
inline __host__ __device__ bool fmt_int4(int fmt) {
  return fmt == CCUT_FMT_AWQ_INT4_G128 || fmt == CCUT_FMT_INT4_SYM_G128;
}

// Byte offset of block (nt, kt, slot) in a packed buffer with `ktiles` k tiles and `nmat`
// interleaved matrices.
inline __host__ __device__ size_t block_offset(int fmt, int nt, int kt, int slot, int ktiles, int nmat) {
  return ((size_t)(nt * ktiles + kt) * nmat + slot) * block_bytes(fmt);
}

// A-tile element of nibble p (AWQ word) -> (row, col) inside the 16x16 tile.
inline __host__ __device__ void awq_nibble_pos(int p, int g, int t, int& row, int& col) {
  row = g + 8 * (p & 1);
  col = 2 * t + (p >> 2) + 8 * ((p >> 1) & 1);
}

// A-tile element of byte b (FP8 k-step) -> (row, col).
inline __host__ __device__ void fp8_byte_pos(int b, int g, int t, int& row, int& col) {
  row = g + 8 * ((b >> 1) & 1);
  col = 2 * t + 8 * (b >> 2) + (b & 1);
}

}  // namespace ccut
