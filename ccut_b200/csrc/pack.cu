// pack.cu -- checkpoint layout -> HBM tile layout, and the fp32 dequant export.
//
// Packing runs once per matrix at load time (the weights then stay resident in HBM); the
// export decodes the packed tiles with the same fragment mapping the GEMM uses, so the
// bit-exact comparison of the export with the CPU dequant also checks the packed layout.
#include "layout.cuh"

namespace ccut {

// AWQ nibble of logical column n in row r of a packed [R, N/8] int32 array.
__device__ __forceinline__ uint32_t awq_get(const int32_t* a, int ncols8, int r, int n, const int* slot_of_col) {
  uint32_t w = static_cast<uint32_t>(a[(size_t)r * ncols8 + (n >> 3)]);
  return (w >> (4 * slot_of_col[n & 7])) & 0xFu;
}

struct NibbleOrder {
  int slot_of_col[8];
};

template <int FMT>  // AWQ or signed int4: the same nibble fragments
__global__ void pack_int4_atoms_kernel(const int32_t* __restrict__ qweight, int K, int N, NibbleOrder ord,
                                       uint8_t* __restrict__ dst, int nmat, int slot) {
  constexpr int kWordsPerBlock = Blk<FMT>::kAtomBytes / 4;
  const int ktiles = K / kTileK;
  const size_t total = (size_t)(N / kTileN) * ktiles * kWordsPerBlock;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int widx = static_cast<int>(i % kWordsPerBlock);
    const size_t blk = i / kWordsPerBlock;
    const int kt = static_cast<int>(blk % ktiles);
    const int nt = static_cast<int>(blk / ktiles);
    const int j = widx & 3;
    const int lane = (widx >> 2) & 31;
    const int kc = (widx >> 7) & 1;
    const int cb = widx >> 8;
    const int g = lane >> 2, t = lane & 3;
    uint32_t word = 0;
#pragma unroll
    for (int p = 0; p < 8; ++p) {
      int row, col;
      awq_nibble_pos(p, g, t, row, col);
      const int n = nt * kTileN + cb * 16 + row;
      const int k = kt * kTileK + kc * 64 + j * 16 + col;
      word |= awq_get(qweight, N / 8, k, n, ord.slot_of_col) << (4 * p);
    }
    uint8_t* b = dst + block_offset(FMT, nt, kt, slot, ktiles, nmat);
    reinterpret_cast<uint32_t*>(b)[widx] = word;
  }
}

// Scales (and AWQ zero points) of channel pair cp of block (nt, kt); `scales` is [K/128, N]
// (fp16 for AWQ, fp32 for the per-channel formats).
template <int FMT>
__device__ __forceinline__ void put_row_meta(uint8_t* b, int r, int n, int kt, int N, const void* scales,
                                             const int32_t* qzeros, const NibbleOrder& ord) {
  using B = Blk<FMT>;
  if constexpr (B::kScale == kScaleF16Row) {
    uint16_t* sc = reinterpret_cast<uint16_t*>(b + B::kScaleOff);
    const uint16_t* src = static_cast<const uint16_t*>(scales);
    sc[r] = src[(size_t)kt * N + n];
    sc[r + 1] = src[(size_t)kt * N + n + 1];
  } else {
    float* sc = reinterpret_cast<float*>(b + B::kScaleOff);
    const float* src = static_cast<const float*>(scales);
    sc[r] = src[(size_t)kt * N + n];
    sc[r + 1] = src[(size_t)kt * N + n + 1];
  }
  if constexpr (B::kZeros) {
    const uint32_t z0 = awq_get(qzeros, N / 8, kt, n, ord.slot_of_col);
    const uint32_t z1 = awq_get(qzeros, N / 8, kt, n + 1, ord.slot_of_col);
    b[B::kZeroOff + (r >> 1)] = static_cast<uint8_t>(z0 | (z1 << 4));
  }
}

// Scale and zero point of row r alone (channel n): the other nibble of the row's zero-point
// byte belongs to the other matrix of a fused block, packed by a separate (earlier or later)
// launch, so the byte is read, modified and written.
template <int FMT>
__device__ __forceinline__ void put_one_row_meta(uint8_t* b, int r, int n, int kt, int N, const void* scales,
                                                 const int32_t* qzeros, const NibbleOrder& ord) {
  using B = Blk<FMT>;
  if constexpr (B::kScale == kScaleF16Row) {
    reinterpret_cast<uint16_t*>(b + B::kScaleOff)[r] = static_cast<const uint16_t*>(scales)[(size_t)kt * N + n];
  } else {
    reinterpret_cast<float*>(b + B::kScaleOff)[r] = static_cast<const float*>(scales)[(size_t)kt * N + n];
  }
  if constexpr (B::kZeros) {
    const uint32_t z = awq_get(qzeros, N / 8, kt, n, ord.slot_of_col);
    uint8_t& zb = b[B::kZeroOff + (r >> 1)];
    zb = static_cast<uint8_t>((zb & (0xF0u >> (4 * (r & 1)))) | (z << (4 * (r & 1))));
  }
}

template <int FMT>  // per-channel metadata of the fragment layout (AWQ and signed int4)
__global__ void pack_int4_meta_kernel(const int32_t* __restrict__ qzeros, const void* __restrict__ scales, int K,
                                      int N, NibbleOrder ord, uint8_t* __restrict__ dst, int nmat, int slot) {
  const int ktiles = K / kTileK;
  const size_t total = (size_t)(N / kTileN) * ktiles * (kTileN / 2);  // one thread per channel pair
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int cp = static_cast<int>(i % (kTileN / 2));
    const size_t blk = i / (kTileN / 2);
    const int kt = static_cast<int>(blk % ktiles);
    const int nt = static_cast<int>(blk / ktiles);
    uint8_t* b = dst + block_offset(FMT, nt, kt, slot, ktiles, nmat);
    put_row_meta<FMT>(b, 2 * cp, nt * kTileN + 2 * cp, kt, N, scales, qzeros, ord);
  }
}

template <int FMT>  // FP8 b128 or channel-scaled
__global__ void pack_fp8_kernel(const uint8_t* __restrict__ w, const float* __restrict__ scale, int K, int N,
                                uint8_t* __restrict__ dst, int nmat, int slot) {
  using B = Blk<FMT>;
  const int ktiles = K / kTileK;
  constexpr int kFragsPerBlock = B::kAtomBytes / 8;  // 8-byte k-step fragments
  const size_t total = (size_t)(N / kTileN) * ktiles * kFragsPerBlock;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int fidx = static_cast<int>(i % kFragsPerBlock);
    const size_t blk = i / kFragsPerBlock;
    const int kt = static_cast<int>(blk % ktiles);
    const int nt = static_cast<int>(blk / ktiles);
    const int j = fidx & 1;
    const int lane = (fidx >> 1) & 31;
    const int kc = (fidx >> 6) & 3;
    const int cb = fidx >> 8;
    const int g = lane >> 2, t = lane & 3;
    uint32_t lo = 0, hi = 0;
#pragma unroll
    for (int bb = 0; bb < 8; ++bb) {
      int row, col;
      fp8_byte_pos(bb, g, t, row, col);
      const int n = nt * kTileN + cb * 16 + row;
      const int k = kt * kTileK + kc * 32 + j * 16 + col;
      const uint32_t v = w[(size_t)n * K + k];
      if (bb < 4) lo |= v << (8 * bb);
      else hi |= v << (8 * (bb - 4));
    }
    uint8_t* b = dst + block_offset(FMT, nt, kt, slot, ktiles, nmat);
    reinterpret_cast<uint2*>(b)[fidx] = make_uint2(lo, hi);
    float* s = reinterpret_cast<float*>(b + B::kScaleOff);
    if constexpr (B::kScale == kScaleF32Row) {  // scale [K/128, N]: channel fidx of the block
      if (fidx < kTileN) s[fidx] = scale[(size_t)kt * N + nt * kTileN + fidx];
    } else if (fidx == 0) {
      s[0] = scale[(size_t)nt * ktiles + kt];
      s[1] = 0.f;
      s[2] = 0.f;
      s[3] = 0.f;
    }
  }
}

// ---- export -------------------------------------------------------------------------
// fp32 scale and zero point of channel (row) c of a packed int4 block.
template <int FMT>
__device__ __forceinline__ void int4_row_meta(const uint8_t* b, int c, float& s, uint32_t& z) {
  using B = Blk<FMT>;
  if constexpr (B::kZeros) {
    z = (b[B::kZeroOff + (c >> 1)] >> (4 * (c & 1))) & 0xF;
    s = __half2float(__ushort_as_half(reinterpret_cast<const uint16_t*>(b + B::kScaleOff)[c]));
  } else {
    z = 8;
    s = reinterpret_cast<const float*>(b + B::kScaleOff)[c];
  }
}

template <int FMT>
__global__ void dequant_int4_kernel(const uint8_t* __restrict__ src, int K, int N, int nmat, int slot,
                                    float* __restrict__ out) {
  using B = Blk<FMT>;
  constexpr int kWordsPerBlock = B::kAtomBytes / 4;
  const int ktiles = K / kTileK;
  const size_t total = (size_t)(N / kTileN) * ktiles * kWordsPerBlock;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int widx = static_cast<int>(i % kWordsPerBlock);
    const size_t blk = i / kWordsPerBlock;
    const int kt = static_cast<int>(blk % ktiles);
    const int nt = static_cast<int>(blk / ktiles);
    const int j = widx & 3, lane = (widx >> 2) & 31, kc = (widx >> 7) & 1, cb = widx >> 8;
    const int g = lane >> 2, t = lane & 3;
    const uint8_t* b = src + block_offset(FMT, nt, kt, slot, ktiles, nmat);
    const uint32_t word = reinterpret_cast<const uint32_t*>(b)[widx];
#pragma unroll
    for (int p = 0; p < 8; ++p) {
      int row, col;
      awq_nibble_pos(p, g, t, row, col);
      const int c = cb * 16 + row;
      const uint32_t q = (word >> (4 * p)) & 0xF;
      float s;
      uint32_t z;
      int4_row_meta<FMT>(b, c, s, z);
      const int n = nt * kTileN + c;
      const int k = kt * kTileK + kc * 64 + j * 16 + col;
      out[(size_t)k * N + n] = __fmul_rn(__fsub_rn((float)q, (float)z), s);
    }
  }
}

template <int FMT>
__global__ void dequant_fp8_kernel(const uint8_t* __restrict__ src, int K, int N, int nmat, int slot,
                                   float* __restrict__ out) {
  using B = Blk<FMT>;
  constexpr int kFragsPerBlock = B::kAtomBytes / 8;
  const int ktiles = K / kTileK;
  const size_t total = (size_t)(N / kTileN) * ktiles * kFragsPerBlock;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int fidx = static_cast<int>(i % kFragsPerBlock);
    const size_t blk = i / kFragsPerBlock;
    const int kt = static_cast<int>(blk % ktiles);
    const int nt = static_cast<int>(blk / ktiles);
    const int j = fidx & 1, lane = (fidx >> 1) & 31, kc = (fidx >> 6) & 3, cb = fidx >> 8;
    const int g = lane >> 2, t = lane & 3;
    const uint8_t* b = src + block_offset(FMT, nt, kt, slot, ktiles, nmat);
    const uint2 frag = reinterpret_cast<const uint2*>(b)[fidx];
    const float* sc = reinterpret_cast<const float*>(b + B::kScaleOff);
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const uint32_t word = r < 2 ? frag.x : frag.y;
      const uint16_t pair = static_cast<uint16_t>(word >> (16 * (r & 1)));
      const uint32_t h2 = e4m3x2_to_f16x2(pair);
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int bb = 2 * r + e;
        int row, col;
        fp8_byte_pos(bb, g, t, row, col);
        const float v = __half2float(__ushort_as_half(static_cast<uint16_t>(h2 >> (16 * e))));
        const int n = nt * kTileN + cb * 16 + row;
        const int k = kt * kTileK + kc * 32 + j * 16 + col;
        const float s = B::kScale == kScaleF32Row ? sc[cb * 16 + row] : sc[0];
        out[(size_t)k * N + n] = __fmul_rn(v, s);
      }
    }
  }
}

// ---- row layout (tcgen05 kernel) ------------------------------------------------------
// Block (nt, kt) of a row-layout buffer sits at (nt * ktiles + kt) * block_bytes; fused
// gate/up buffers (nmat = 2) hold both matrices in every block.
template <int FMT>
__global__ void pack_int4_rows_kernel(const int32_t* __restrict__ qweight, const int32_t* __restrict__ qzeros,
                                      const void* __restrict__ scales, int K, int N, NibbleOrder ord,
                                      uint8_t* __restrict__ dst, int nmat, int slot) {
  using B = Blk<FMT>;
  constexpr int kWordsPerRow = kTileK / 8;  // 16
  const int ktiles = K / kTileK, nblk = rows_nblocks(N, nmat);
  const size_t total = (size_t)nblk * ktiles * kTileN * (kWordsPerRow + 1);
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int widx = static_cast<int>(i % (kTileN * (kWordsPerRow + 1)));
    const size_t blk = i / (kTileN * (kWordsPerRow + 1));
    const int kt = static_cast<int>(blk % ktiles);
    const int nt = static_cast<int>(blk / ktiles);
    const int r = widx / (kWordsPerRow + 1), j = widx % (kWordsPerRow + 1);
    const int n = rows_channel(nt, r, nmat, slot);
    if (n < 0) continue;
    uint8_t* b = dst + ((size_t)nt * ktiles + kt) * B::kBytes;
    if (j < kWordsPerRow) {
      uint32_t word = 0;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const int k = kt * kTileK + 8 * j + kk;
        word |= awq_get(qweight, N / 8, k, n, ord.slot_of_col) << (4 * rows_awq_slot(kk));
      }
      *reinterpret_cast<uint32_t*>(b + rows_awq_word(r, 8 * j)) = word;
    } else if (nmat == 2) {  // fused: row r alone is this matrix's (rows alternate gate / up)
      put_one_row_meta<FMT>(b, r, n, kt, N, scales, qzeros, ord);
    } else if ((r & 1) == 0) {  // metadata of rows r, r + 1 (zero points share a byte)
      put_row_meta<FMT>(b, r, n, kt, N, scales, qzeros, ord);
    }
  }
}

template <int FMT>
__global__ void pack_fp8_rows_kernel(const uint8_t* __restrict__ w, const float* __restrict__ scale, int K, int N,
                                     uint8_t* __restrict__ dst, int nmat, int slot) {
  using B = Blk<FMT>;
  constexpr int kChunksPerRow = kTileK / 16;  // 8
  const int ktiles = K / kTileK, nblk = rows_nblocks(N, nmat);
  const size_t total = (size_t)nblk * ktiles * kTileN * kChunksPerRow;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int cidx = static_cast<int>(i % (kTileN * kChunksPerRow));
    const size_t blk = i / (kTileN * kChunksPerRow);
    const int kt = static_cast<int>(blk % ktiles);
    const int nt = static_cast<int>(blk / ktiles);
    const int r = cidx >> 3, c = cidx & 7;
    const int n = rows_channel(nt, r, nmat, slot);
    if (n < 0) continue;
    const uint4 v = *reinterpret_cast<const uint4*>(w + (size_t)n * K + kt * kTileK + 16 * c);
    uint8_t* b = dst + ((size_t)nt * ktiles + kt) * B::kBytes;
    *reinterpret_cast<uint4*>(b + rows_fp8_byte(r, 16 * c)) = v;
    if constexpr (B::kScale == kScaleF32Row) {  // scale [K/128, N]: the row's channel
      if (c == 0) reinterpret_cast<float*>(b + B::kScaleOff)[r] = scale[(size_t)kt * N + n];
    } else if (c == 0 && (nmat == 2 ? r == slot : r == 0)) {
      // block scale(s): a fused gate/up block keeps the gate scale at [0], the up scale at [1]
      float* s = reinterpret_cast<float*>(b + B::kScaleOff);
      s[nmat == 2 ? slot : 0] = scale[(size_t)(n / 128) * ktiles + kt];
      if (slot == 0) {
        if (nmat == 1) s[1] = 0.f;
        s[2] = 0.f;
        s[3] = 0.f;
      }
    }
  }
}

template <int FMT>
__global__ void dequant_int4_rows_kernel(const uint8_t* __restrict__ src, int K, int N, int nmat, int slot,
                                         float* __restrict__ out) {
  using B = Blk<FMT>;
  constexpr int kWordsPerRow = kTileK / 8;
  const int ktiles = K / kTileK, nblk = rows_nblocks(N, nmat);
  const size_t total = (size_t)nblk * ktiles * kTileN * kWordsPerRow;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int widx = static_cast<int>(i % (kTileN * kWordsPerRow));
    const size_t blk = i / (kTileN * kWordsPerRow);
    const int kt = static_cast<int>(blk % ktiles);
    const int nt = static_cast<int>(blk / ktiles);
    const int r = widx / kWordsPerRow, j = widx % kWordsPerRow;
    const int n = rows_channel(nt, r, nmat, slot);
    if (n < 0) continue;
    const uint8_t* b = src + ((size_t)nt * ktiles + kt) * B::kBytes;
    const uint32_t word = *reinterpret_cast<const uint32_t*>(b + rows_awq_word(r, 8 * j));
    float s;
    uint32_t z;
    int4_row_meta<FMT>(b, r, s, z);
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      const uint32_t q = (word >> (4 * rows_awq_slot(kk))) & 0xF;
      const int k = kt * kTileK + 8 * j + kk;
      out[(size_t)k * N + n] = __fmul_rn(__fsub_rn((float)q, (float)z), s);
    }
  }
}

template <int FMT>
__global__ void dequant_fp8_rows_kernel(const uint8_t* __restrict__ src, int K, int N, int nmat, int slot,
                                        float* __restrict__ out) {
  using B = Blk<FMT>;
  constexpr int kChunksPerRow = kTileK / 16;
  const int ktiles = K / kTileK, nblk = rows_nblocks(N, nmat);
  const size_t total = (size_t)nblk * ktiles * kTileN * kChunksPerRow;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int cidx = static_cast<int>(i % (kTileN * kChunksPerRow));
    const size_t blk = i / (kTileN * kChunksPerRow);
    const int kt = static_cast<int>(blk % ktiles);
    const int nt = static_cast<int>(blk / ktiles);
    const int r = cidx >> 3, c = cidx & 7;
    const int n = rows_channel(nt, r, nmat, slot);
    if (n < 0) continue;
    const uint8_t* b = src + ((size_t)nt * ktiles + kt) * B::kBytes;
    const uint4 v = *reinterpret_cast<const uint4*>(b + rows_fp8_byte(r, 16 * c));
    const float s = reinterpret_cast<const float*>(b + B::kScaleOff)[B::kScale == kScaleF32Row ? r
                                                                      : nmat == 2                  ? slot
                                                                                                   : 0];
    const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const uint32_t h2 = e4m3x2_to_f16x2(static_cast<uint16_t>(w4[q >> 1] >> (16 * (q & 1))));
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int k = kt * kTileK + 16 * c + 2 * q + e;
        const float val = __half2float(__ushort_as_half(static_cast<uint16_t>(h2 >> (16 * e))));
        out[(size_t)k * N + n] = __fmul_rn(val, s);
      }
    }
  }
}

static int grid_for(size_t total, int threads) {
  size_t g = (total + threads - 1) / threads;
  if (g > 148 * 32) g = 148 * 32;
  return static_cast<int>(g < 1 ? 1 : g);
}

static NibbleOrder make_order(int nibble_order) {
  NibbleOrder o;
  static const int awq_slot_of_col[8] = {0, 4, 1, 5, 2, 6, 3, 7};  // column c lives in slot [c]
  for (int c = 0; c < 8; ++c) o.slot_of_col[c] = nibble_order == CCUT_NIBBLES_AWQ ? awq_slot_of_col[c] : c;
  return o;
}

template <int FMT>
static void launch_pack_t(int layout, const void* q, const void* z, const void* s, int K, int N, int nibble_order,
                          uint8_t* dst, int nmat, int slot, cudaStream_t st) {
  const int threads = 256;
  const int ktiles = K / kTileK, ntiles = N / kTileN;
  const int32_t* qw = static_cast<const int32_t*>(q);
  const int32_t* qz = static_cast<const int32_t*>(z);
  if (layout == kLayoutRows) {
    const int nblk = rows_nblocks(N, nmat);
    if constexpr (Blk<FMT>::kInt4) {
      const size_t t1 = (size_t)nblk * ktiles * kTileN * 17;
      pack_int4_rows_kernel<FMT><<<grid_for(t1, threads), threads, 0, st>>>(qw, qz, s, K, N, make_order(nibble_order),
                                                                            dst, nmat, slot);
    } else {
      const size_t t1 = (size_t)nblk * ktiles * kTileN * 8;
      pack_fp8_rows_kernel<FMT><<<grid_for(t1, threads), threads, 0, st>>>(
          static_cast<const uint8_t*>(q), static_cast<const float*>(s), K, N, dst, nmat, slot);
    }
  } else if constexpr (Blk<FMT>::kInt4) {
    const NibbleOrder o = make_order(nibble_order);
    const size_t t1 = (size_t)ntiles * ktiles * (Blk<FMT>::kAtomBytes / 4);
    pack_int4_atoms_kernel<FMT><<<grid_for(t1, threads), threads, 0, st>>>(qw, K, N, o, dst, nmat, slot);
    const size_t t2 = (size_t)ntiles * ktiles * (kTileN / 2);
    pack_int4_meta_kernel<FMT><<<grid_for(t2, threads), threads, 0, st>>>(qz, s, K, N, o, dst, nmat, slot);
  } else {
    const size_t t1 = (size_t)ntiles * ktiles * (Blk<FMT>::kAtomBytes / 8);
    pack_fp8_kernel<FMT><<<grid_for(t1, threads), threads, 0, st>>>(
        static_cast<const uint8_t*>(q), static_cast<const float*>(s), K, N, dst, nmat, slot);
  }
}

int launch_pack(int fmt, int layout, const void* q, const void* z, const void* s, int K, int N, int nibble_order,
                void* dst, int nmat, int slot, cudaStream_t st) {
  uint8_t* d = static_cast<uint8_t*>(dst);
  switch (fmt) {
    case CCUT_FMT_AWQ_INT4_G128:
      launch_pack_t<CCUT_FMT_AWQ_INT4_G128>(layout, q, z, s, K, N, nibble_order, d, nmat, slot, st);
      break;
    case CCUT_FMT_INT4_SYM_G128:
      launch_pack_t<CCUT_FMT_INT4_SYM_G128>(layout, q, z, s, K, N, nibble_order, d, nmat, slot, st);
      break;
    case CCUT_FMT_FP8_E4M3_CH:
      launch_pack_t<CCUT_FMT_FP8_E4M3_CH>(layout, q, z, s, K, N, nibble_order, d, nmat, slot, st);
      break;
    default:
      launch_pack_t<CCUT_FMT_FP8_E4M3_B128>(layout, q, z, s, K, N, nibble_order, d, nmat, slot, st);
  }
  return cudaPeekAtLastError() == cudaSuccess ? CCUT_OK : CCUT_ERR_CUDA;
}

template <int FMT>
static void launch_dequant_t(int layout, const uint8_t* packed, int K, int N, int nmat, int slot, float* out,
                             cudaStream_t st) {
  const int threads = 256;
  const int ktiles = K / kTileK, ntiles = N / kTileN;
  if (layout == kLayoutRows) {
    const int nblk = rows_nblocks(N, nmat);
    if constexpr (Blk<FMT>::kInt4) {
      const size_t t = (size_t)nblk * ktiles * kTileN * 16;
      dequant_int4_rows_kernel<FMT><<<grid_for(t, threads), threads, 0, st>>>(packed, K, N, nmat, slot, out);
    } else {
      const size_t t = (size_t)nblk * ktiles * kTileN * 8;
      dequant_fp8_rows_kernel<FMT><<<grid_for(t, threads), threads, 0, st>>>(packed, K, N, nmat, slot, out);
    }
  } else if constexpr (Blk<FMT>::kInt4) {
    const size_t t = (size_t)ntiles * ktiles * (Blk<FMT>::kAtomBytes / 4);
    dequant_int4_kernel<FMT><<<grid_for(t, threads), threads, 0, st>>>(packed, K, N, nmat, slot, out);
  } else {
    const size_t t = (size_t)ntiles * ktiles * (Blk<FMT>::kAtomBytes / 8);
    dequant_fp8_kernel<FMT><<<grid_for(t, threads), threads, 0, st>>>(packed, K, N, nmat, slot, out);
  }
}

int launch_dequant(int fmt, int layout, const void* packed, int K, int N, int nmat, int slot, float* out,
                   cudaStream_t st) {
  const uint8_t* p = static_cast<const uint8_t*>(packed);
  switch (fmt) {
    case CCUT_FMT_AWQ_INT4_G128:
      launch_dequant_t<CCUT_FMT_AWQ_INT4_G128>(layout, p, K, N, nmat, slot, out, st);
      break;
    case CCUT_FMT_INT4_SYM_G128:
      launch_dequant_t<CCUT_FMT_INT4_SYM_G128>(layout, p, K, N, nmat, slot, out, st);
      break;
    case CCUT_FMT_FP8_E4M3_CH:
      launch_dequant_t<CCUT_FMT_FP8_E4M3_CH>(layout, p, K, N, nmat, slot, out, st);
      break;
    default:
      launch_dequant_t<CCUT_FMT_FP8_E4M3_B128>(layout, p, K, N, nmat, slot, out, st);
  }
  return cudaPeekAtLastError() == cudaSuccess ? CCUT_OK : CCUT_ERR_CUDA;
}

}  // namespace ccut
