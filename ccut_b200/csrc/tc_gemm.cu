// tc_gemm.cu -- tcgen05 dequant-fused grouped expert GEMM (gate/up + SiLU, and down) on
// pairs of SMs.
//
// Swap-AB formulation over a CTA pair (cta_group::2): the 256 rows of two weight blocks are
// the MMA's M dimension (A operand, rank 0 holds block 2p, rank 1 block 2p + 1), the N <= 256
// tokens of a row tile are N (B operand, each rank holds N/2 of them), and D lives in tensor
// memory (each rank: its 128 weight rows x all N tokens):
//   D[row, token] (+)= A[row, k] * B[token, k]     (tcgen05.mma.cta_group::2.kind::f16, M=256)
// Measured on B200: an M=128, K=16 MMA costs ~118 clk at any N <= 192 and ~138 at N = 256,
// so tiles are as wide as the expert's rows allow (up to 256); with both operands in shared
// memory a single SM reads 12 KB per N=256 MMA and slows to ~171 clk, while the pair splits
// that to 8 KB per SM.
//
// Exact operands.  The A operand is the quantized weight itself in bf16: q - z for AWQ (an
// integer in [-15, 15]) and the e4m3 value for FP8, both exact; activations are the bf16
// inputs (gathered in expert order) and the bf16 SwiGLU rows.  Each 128-k block (one AWQ group
// / one FP8 scale block) accumulates into a partial sum in tensor memory, and the epilogue
// warps promote it into fp32 totals in registers with the block's fp32 scale:
//   total[row, token] += s[row, kb] * partial_kb[row, token]
// which is the reference's dequantize-then-multiply (w = (q - z) * s, or e4m3 * s, in fp32)
// reassociated in fp32.  Two partial buffers of 256 columns (all 512 tensor-memory columns)
// let the MMAs of block kb + 1 run while block kb is promoted.
//
// Work item = (expert, token tile of up to 256 rows, pair p of 128-row weight blocks); cluster
// c takes item c, then the items a launch-wide counter hands out (warp 3 of rank 0 claims
// them and passes them to every role of both CTAs through a small ring).  A 64-k stage is
// one A tile (128 rows x 64 k bf16, 16 KB) and one B tile (128 tokens x 64 k, 16 KB) per CTA.
// Warp roles (20 warps per CTA):
//   warp 0        weight producer: per stage one bulk copy of the packed 64-k half block (and
//                 its scale / zero-point metadata) into the weight ring
//   warp 1        activation producer: one TMA tile per stage, counted on rank 0's barrier
//   warp 2        rank 0: the MMA issuer (one thread); both ranks: tensor-memory allocation
//   warps 4..11   two dequant warpgroups: one weight row and 32 k of each stage per thread,
//                 into the A tile (128-byte swizzled K-major), then a proxy fence and an
//                 arrival on rank 0's barrier
//   warps 12..19  two epilogue warpgroups (128 token columns each): promotion of every 128-k
//                 partial (packed fp32x2 FMAs), then silu(gate) * up as bf16 rows (gate rows
//                 pair with up rows through shared memory) or row_weight * total as fp32 rows
// Registers: warpgroups 0 to 2 give theirs up (setmaxnreg) so that each epilogue thread can
// hold its 128 fp32 totals.  Every wait is bounded; an expired wait records CCUT_ERR_TIMEOUT
// and the kernel unwinds.
//
// Follows ccut/blocks/moe.py:122-141 (expert_ffn), ccut/quant/kernels.py:219-231 (SiLU),
// the dequant of ccut/quant/kernels.py:150-171 / :276-295 (restated for the group-128 /
// block-128 formats) and ccut/models/generic.py:377-378 (routing-weight scaling).
#include <stdlib.h>

#include "kernels.cuh"
#include "tc.cuh"

namespace ccut {

// Work items reach every role of both CTAs through a ring of kItemRing slots that rank 0's
// scheduler thread fills; each slot is freed by all its consumers: per CTA the two producer
// threads and every dequant and epilogue warp, plus the MMA issuer of rank 0.
constexpr int kItemRing = 4;
constexpr int kItemConsumers = 2 * (2 + 8 + 8) + 1;

template <int FMT>
struct TcCfg {
  using B = Blk<FMT>;
  static constexpr bool kInt4 = B::kInt4;
  static constexpr int kMaxN = 256;                   // tokens per tile (both ranks)
  static constexpr int kHalfW = kInt4 ? 4096 : 8192;  // packed weights of one 64-k half block
  // Metadata copied with each stage: AWQ scales + zero points (the dequant reads the zero
  // points), the per-channel fp32 scales, the FP8 block scale slot; this also brings the
  // scales the epilogue reads into L2.
  static constexpr int kMeta = B::kScale == kScaleF32Row ? 512 : B::kZeros ? 320 : 16;
  static constexpr int kWBytes = kHalfW + kMeta;      // one weight stage (multiple of 16)
  static constexpr int kAB = 32768;                   // A tile 16 KB + B tile 16 KB
  static constexpr int kSA = 5;                       // A/B stages
  static constexpr int kSW = kInt4 ? 6 : 4;           // weight stages
  static constexpr int kXRow = 17;                    // FFN1 staging: floats per weight row (16 + pad)
  static constexpr int kTokPitch = 132;               // FFN2 staging: floats per token (128 + pad, 16-B rows)
  // FFN1 staging (bf16 elements): 16 token rows of 64 channels for the even lanes' tokens, then
  // (after 64 bytes of padding, so that the odd lanes' stores hit other banks) the odd lanes'
  static constexpr int kFfn1Odd = 16 * 64 + 32;
  static constexpr int kFfn1Buf = kFfn1Odd + 16 * 64;
  static constexpr int kXchg = 2 * 128 * kXRow * 4;   // per epilogue warpgroup: 128 rows x 16 tokens
  static_assert(16 * kTokPitch <= 128 * kXRow && (kTokPitch * 4) % 16 == 0, "FFN2 staging fits the exchange");
  static_assert(2 * kFfn1Buf * 2 <= 128 * kXRow * 4 && (kFfn1Buf * 2) % 16 == 0, "FFN1 staging fits the exchange");
  static constexpr int kThreads = 640;
  static constexpr int kDeqWarps = 8;
  static constexpr int kEpiWarps = 8;
  static_assert(kItemConsumers == 2 * (2 + kDeqWarps + kEpiWarps) + 1, "item ring consumers");
  static constexpr int kNBar = 2 * kSW + 2 * kSA + 2 + 2 + 1 + 2 * kItemRing + 1;
  // barriers, tensor-memory address, item prefix over experts, the experts' row offsets and
  // tile descriptors
  static constexpr int kHeader = kNBar * 8 + 16 + 3 * 4 * (kMaxExperts + 1) + 4 * kItemRing;
  static constexpr int kXchgOff = (kHeader + 1023) / 1024 * 1024;
  static constexpr int kRowWOff = kXchgOff + kXchg;   // FFN2: routing weights of the item's 256 tokens
  static constexpr int kABOff = kXchgOff + (kXchg + 256 * 4 + 1023) / 1024 * 1024;  // 1024-aligned tiles
  static constexpr int kWOff = kABOff + kSA * kAB;
  static constexpr int kSmem = kWOff + kSW * kWBytes + 1024;  // +1024: runtime alignment slack
  static_assert(kSmem <= 227 * 1024, "shared memory budget");
  static_assert(kWBytes % 16 == 0, "bulk copies move multiples of 16 bytes");
};

// Register shares after setmaxnreg (multiples of 8): the launch gives 640 threads x 96 (the
// largest multiple of 8 within 65536 / 640).
constexpr uint32_t kRegProducers = 32, kRegDequant = 48, kRegEpilogue = 176;
static_assert(128 * kRegProducers + 256 * kRegDequant + 256 * kRegEpilogue <= 640 * 96, "register pool");

// Item -> (expert e, weight block pair p, first tile row m0, rows, tile width N).  An expert's
// M_e rows are cut into ceil(M_e / 256) tiles of equal width (a multiple of 32); tdesc[e]
// holds that width << 16 | the tile count (set up once per CTA, so a decode is a binary
// search plus a few shared-memory reads, without integer divisions for 1 or 2 tiles).
__device__ __forceinline__ void tc_decode_item(int item, const int* tprefix, int num_e, const int* offsets,
                                               const int* tdesc, int& e, int& p, int& m0, int& rows, int& n) {
  int lo = 0, hi = num_e - 1;  // last e with tprefix[e] <= item
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (tprefix[mid] <= item) lo = mid;
    else hi = mid - 1;
  }
  e = lo;
  const int d = tdesc[e], mtiles = d & 0xffff, tw = d >> 16;
  const int local = item - tprefix[e];
  int mt;
  if (mtiles == 1) {
    p = local;
    mt = 0;
  } else if (mtiles == 2) {
    p = local >> 1;
    mt = local & 1;
  } else {
    p = local / mtiles;
    mt = local - p * mtiles;
  }
  m0 = mt * tw;
  rows = min(tw, offsets[e + 1] - offsets[e] - m0);
  n = (rows + 31) / 32 * 32;
}

__device__ __forceinline__ uint32_t bf16x2_sub(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
// Bytes `sel` of a word of e4m3 codes -> bf16x2 with integer / bf16 FMA-pipe operations only
// (the conversion pipe is left to the epilogue's exp / reciprocal).  The code's 7 magnitude
// bits placed at bf16 bits [10:4] read as e4m3 * 2^-120 (exponent field E, mantissa M; for
// E = 0 a bf16 subnormal 0.M * 2^-126, again e4m3 * 2^-120), so one bf16 multiply by +-2^120,
// carrying the sign, gives the e4m3 value exactly, subnormals and zeros included.  The two
// NaN codes (0x7F, 0xFF) come out as +-480: valid FP8 checkpoints do not hold them (the debug
// export and the mma.sync kernel keep them NaN).
template <uint32_t kSel>  // prmt selector placing the two codes at bits [15:8] and [31:24]
__device__ __forceinline__ uint32_t e4m3x2_to_bf16x2(uint32_t w) {
  uint32_t x, mag, sgn, r;
  asm("prmt.b32 %0, %1, 0, %2;" : "=r"(x) : "r"(w), "n"(kSel));
  asm("shr.b32 %0, %1, 4;" : "=r"(mag) : "r"(x));
  asm("and.b32 %0, %1, 0x07F007F0;" : "=r"(mag) : "r"(mag));
  asm("lop3.b32 %0, %1, 0x80008000, 0x7B807B80, 0xEA;" : "=r"(sgn) : "r"(x));  // (x & 0x80008000) | 2^120
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(mag), "r"(sgn));
  return r;
}

// k [32 h, 32 h + 32) of row r of a staged 64-k half block -> 32 bf16 weights (unscaled) in
// row r of the A tile, 128-byte swizzled K-major: 16-byte chunk c (k 8c .. 8c + 7) at
// r * 128 + ((c ^ (r & 7)) << 4).
template <int FMT>
__device__ __forceinline__ void dequant_half_row(const uint8_t* half, const uint8_t* zeros, int r, int h,
                                                 uint8_t* atile) {
  uint8_t* arow = atile + r * 128;
  if constexpr (!Blk<FMT>::kInt4) {
#pragma unroll
    for (int cc = 0; cc < 2; ++cc) {  // 16 e4m3 values: k 16c .. 16c + 15
      const int c = 2 * h + cc;
      const uint4 q = *reinterpret_cast<const uint4*>(half + r * 64 + 16 * (c ^ ((r >> 1) & 3)));
      const uint32_t w4[4] = {q.x, q.y, q.z, q.w};
      uint32_t o[8];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        o[2 * i] = e4m3x2_to_bf16x2<0x1404>(w4[i]);      // bytes 0, 1
        o[2 * i + 1] = e4m3x2_to_bf16x2<0x3424>(w4[i]);  // bytes 2, 3
      }
      *reinterpret_cast<uint4*>(arow + (((2 * c) ^ (r & 7)) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
      *reinterpret_cast<uint4*>(arow + (((2 * c + 1) ^ (r & 7)) << 4)) = make_uint4(o[4], o[5], o[6], o[7]);
    }
  } else {
    const uint32_t z = Blk<FMT>::kZeros ? (zeros[r >> 1] >> (4 * (r & 1))) & 0xFu : 8u;
    const uint32_t zz = (0x4300u | z) * 0x10001u;  // bf16x2 (128 + z, 128 + z)
    const uint4 q = *reinterpret_cast<const uint4*>(half + r * 32 + 16 * (h ^ ((r >> 2) & 1)));  // k 32h .. +31
    const uint32_t w4[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {  // word j: k 32h + 8j .. +7 -> A chunk 4h + j
      uint32_t o[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        uint32_t v;  // bf16x2 (128 + q_lo, 128 + q_hi); minus (128 + z) is q - z, exact
        asm("lop3.b32 %0, %1, 0x000F000F, 0x43004300, 0xEA;" : "=r"(v) : "r"(w4[j] >> (4 * i)));
        o[i] = bf16x2_sub(v, zz);
      }
      *reinterpret_cast<uint4*>(arow + (((4 * h + j) ^ (r & 7)) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
}

// fp32 scale of weight row r of the block at `blk` (one 128-k block).
template <int FMT, int MODE>
__device__ __forceinline__ float block_scale(const uint8_t* blk, int r) {
  using B = Blk<FMT>;
  if constexpr (B::kScale == kScaleF16Row) {
    return __half2float(__ushort_as_half(__ldg(reinterpret_cast<const unsigned short*>(blk + B::kScaleOff) + r)));
  } else if constexpr (B::kScale == kScaleF32Row) {
    return __ldg(reinterpret_cast<const float*>(blk + B::kScaleOff) + r);
  } else {
    return __ldg(reinterpret_cast<const float*>(blk + B::kScaleOff) + (MODE == kFfn1 ? (r & 1) : 0));
  }
}

// The u-th work item of this CTA's walk from the item ring (one thread), its slot freed on
// rank 0: an item id, -1 at the end of the walk, -2 when the wait ran out.
__device__ __forceinline__ int tc_ring_item(int u, uint64_t* ifull, const int* iring, uint64_t* iempty, int* status) {
  const int slot = u % kItemRing;
  if (!tc::mbar_wait_cl(&ifull[slot], (u / kItemRing) & 1, status)) return -2;
  const int item = *reinterpret_cast<const volatile int*>(&iring[slot]);
  tc::mbar_arrive_cl(tc::mapa(&iempty[slot], 0));
  return item;
}
// The same for a whole warp: lane 0 takes the slot, every lane gets the item.
__device__ __forceinline__ int tc_ring_item_warp(int u, uint64_t* ifull, const int* iring, uint64_t* iempty,
                                                 int* status, int lane) {
  int item = 0;
  if (lane == 0) item = tc_ring_item(u, ifull, iring, iempty, status);
  return __shfl_sync(0xffffffffu, item, 0);
}

__device__ __forceinline__ void named_bar(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// total[i] += s * partial[i] for 16 columns, as 8 packed fp32x2 FMAs.
__device__ __forceinline__ void promote16(float* tot, const uint32_t (&v)[16], float s) {
  const uint64_t ss = (static_cast<uint64_t>(__float_as_uint(s)) << 32) | __float_as_uint(s);
#pragma unroll
  for (int i = 0; i < 16; i += 2) {
    uint64_t acc = (static_cast<uint64_t>(__float_as_uint(tot[i + 1])) << 32) | __float_as_uint(tot[i]);
    const uint64_t pv = (static_cast<uint64_t>(v[i + 1]) << 32) | v[i];
    asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(acc) : "l"(ss), "l"(pv));
    tot[i] = __uint_as_float(static_cast<uint32_t>(acc));
    tot[i + 1] = __uint_as_float(static_cast<uint32_t>(acc >> 32));
  }
}

template <int FMT, int MODE>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(640, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap bmap, TcArgs a) {
  pdl_wait();
  pdl_trigger();
  using C = TcCfg<FMT>;
  using BK = Blk<FMT>;
  constexpr int SA = C::kSA;
  constexpr int SW = C::kSW;
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte alignment for the 128-byte-swizzled operand tiles (the same offset in both CTAs)
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem);
  uint64_t* wfull = bars;           // [SW] weight stage landed
  uint64_t* wempty = wfull + SW;    // [SW] weight stage converted
  uint64_t* abfull = wempty + SW;   // [SA] rank 0: A and B tiles of both CTAs ready
  uint64_t* abempty = abfull + SA;  // [SA] MMAs of the stage done (committed to both CTAs)
  uint64_t* pfull = abempty + SA;   // [2] partial sums of a 128-k block ready (both CTAs)
  uint64_t* pempty = pfull + 2;     // [2] rank 0: partial buffer drained by both CTAs
  uint64_t* drain = pempty + 2;
  uint64_t* ifull = drain + 1;              // [kItemRing] item slot written (both CTAs)
  uint64_t* iempty = ifull + kItemRing;     // [kItemRing] rank 0: item slot read by every consumer
  uint64_t* idemand = iempty + kItemRing;   // rank 0: its weight producer took the next item
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + C::kNBar);
  int* tprefix = reinterpret_cast<int*>(smem + C::kNBar * 8 + 16);
  int* soff = tprefix + kMaxExperts + 1;  // a.offsets, read once: every role decodes items from it
  int* tdesc = soff + kMaxExperts + 1;    // per expert: tile width << 16 | tile count
  int* iring = tdesc + kMaxExperts + 1;   // [kItemRing] work item ids (-1: end of the walk)
  float* xchg = reinterpret_cast<float*>(smem + C::kXchgOff);
  uint8_t* ab = smem + C::kABOff;
  uint8_t* wtiles = smem + C::kWOff;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = tc::cluster_rank();
  const int cluster = blockIdx.x >> 1, nclusters = gridDim.x >> 1;
  const int ntiles = a.N / kTileN, npairs = (ntiles + 1) / 2;
  const int ktiles = a.K / kTileK, nstages = a.K / 64, nkb = ktiles;

  if (warp == 2) {
    tc::tmem_alloc2(tmem_slot, 512);
    tc::tmem_relinquish2();
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < SW; ++s) {
      mbar_init(&wfull[s], 1);
      mbar_init(&wempty[s], C::kDeqWarps);
    }
    for (int s = 0; s < SA; ++s) {
      mbar_init(&abfull[s], 2 * C::kDeqWarps + 2);  // dequant warps of both CTAs + both TMA threads
      mbar_init(&abempty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&pfull[i], 1);
      mbar_init(&pempty[i], 2 * C::kEpiWarps);
    }
    mbar_init(drain, 1);
    for (int i = 0; i < kItemRing; ++i) {
      mbar_init(&ifull[i], 1);
      mbar_init(&iempty[i], kItemConsumers);
    }
    mbar_init(idemand, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    tc::prefetch_tmap(&bmap);
  }
  if (warp == 3) {  // item prefix over experts: items(e) = ceil(M_e / 256) * npairs
    int carry = 0;
    for (int b = 0; b < a.num_e; b += 32) {
      const int e = b + lane;
      const int o0 = e < a.num_e ? a.offsets[e] : 0, o1 = e < a.num_e ? a.offsets[e + 1] : 0;
      if (e < a.num_e) soff[e] = o0;
      if (e == a.num_e - 1) soff[e + 1] = o1;
      const int me = o1 - o0;
      const int mt = (me + 255) / 256;
      if (e < a.num_e) tdesc[e] = (mt > 0 ? ((me + mt - 1) / mt + 31) / 32 * 32 : 0) << 16 | mt;
      const int c = mt * npairs;
      int inc = c;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int u = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += u;
      }
      if (e < a.num_e) tprefix[e] = carry + inc - c;
      carry += __shfl_sync(0xffffffffu, inc, 31);
    }
    if (lane == 0) tprefix[a.num_e] = carry;
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::cluster_sync();  // the peer's barriers are initialised before any remote arrival
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  const int total = tprefix[a.num_e];

  if (warp < 4) {
    tc::setmaxnreg_dec<kRegProducers>();
    if (warp == 0 && lane == 0) {
      // ------------------------------------------------------------ weight producer
      int use = 0;
      bool ok = true;
      for (int iu = 0; ok; ++iu) {
        const int item = tc_ring_item(iu, ifull, iring, iempty, a.status);
        if (item < 0) {
          ok = item == -1;
          break;
        }
        if (rank == 0) mbar_arrive(idemand);  // the scheduler may claim the item after this one
        int e, p, m0, rows, n;
        tc_decode_item(item, tprefix, a.num_e, soff, tdesc, e, p, m0, rows, n);
        const int blk = 2 * p + (int)rank;
        const bool valid = blk < ntiles;
        const uint8_t* wb = a.w + (size_t)e * a.expert_stride + (size_t)(valid ? blk : 0) * ktiles * BK::kBytes;
        for (int st = 0; st < nstages; ++st, ++use) {
          const int s = use % SW;
          // a suspending wait: a spinning warp would take issue slots from the dequant warp
          // that shares its SM sub-partition
          if (!mbar_wait(&wempty[s], ((use / SW) & 1) ^ 1, a.status)) {
            ok = false;
            break;
          }
          if (valid) {
            uint8_t* sb = wtiles + s * C::kWBytes;
            const uint8_t* blkp = wb + (size_t)(st >> 1) * BK::kBytes;
            mbar_arrive_expect_tx(&wfull[s], C::kWBytes);
            bulk_g2s(sb, blkp + (st & 1) * C::kHalfW, C::kHalfW, &wfull[s]);
            bulk_g2s(sb + C::kHalfW, blkp + BK::kScaleOff, C::kMeta, &wfull[s]);
          } else {
            mbar_arrive(&wfull[s]);
          }
        }
      }
      if (!ok)  // let issued copies land before the CTA exits
        for (int u = use > SW ? use - SW : 0; u < use; ++u) mbar_wait(&wfull[u % SW], (u / SW) & 1, nullptr);
    } else if (warp == 1 && lane == 0) {
      // ------------------------------------------------------------ activation producer
      int use = 0;
      bool ok = true;
      for (int iu = 0; ok; ++iu) {
        const int item = tc_ring_item(iu, ifull, iring, iempty, a.status);
        if (item < 0) {
          ok = item == -1;
          break;
        }
        int e, p, m0, rows, n;
        tc_decode_item(item, tprefix, a.num_e, soff, tdesc, e, p, m0, rows, n);
        const int brow = soff[e] + m0 + (int)rank * (n / 2);
        for (int st = 0; st < nstages; ++st, ++use) {
          const int sa = use % SA;
          if (!tc::mbar_wait_cl(&abempty[sa], ((use / SA) & 1) ^ 1, a.status)) {
            ok = false;
            break;
          }
          const uint32_t bar0 = tc::mapa(&abfull[sa], 0);
          tc::mbar_arrive_expect_tx_cl(bar0, 16384);
          tc::tma_load_2d_pair(ab + sa * C::kAB + 16384, &bmap, st * 64, brow, bar0);
        }
      }
      if (!ok)  // let issued loads land: the last stage's MMAs (or the timeout) end them
        for (int u = use > SA ? use - SA : 0; u < use; ++u) tc::mbar_wait_cl(&abempty[u % SA], (u / SA) & 1, nullptr);
    } else if (warp == 3 && lane == 0 && rank == 0) {
      // ------------------------------------------------------------ item scheduler (rank 0)
      // Cluster c walks item c first, then (a.sched) the items a launch-wide counter hands
      // out, so that clusters whose items ran faster take more and the SMs end together, or
      // (no counter) c + nclusters, c + 2 nclusters, ...  An item is claimed only once rank
      // 0's weight producer has taken the one before it, so a cluster holds at most one
      // claimed item it has not started.  -1 ends the walk.
      const uint32_t peer_ring = tc::mapa(iring, 1);
      for (int u = 0;; ++u) {
        const int slot = u % kItemRing;
        if (!tc::mbar_wait_cl(&iempty[slot], ((u / kItemRing) & 1) ^ 1, a.status)) break;
        if (u > 0 && !mbar_wait(idemand, (u - 1) & 1, a.status)) break;
        int item = u == 0 ? cluster : a.sched ? nclusters + atomicAdd(&a.sched[0], 1) : cluster + u * nclusters;
        if (item >= total) item = -1;
        iring[slot] = item;
        tc::st_cluster_u32(peer_ring + 4 * slot, (uint32_t)item);
        tc::mbar_arrive_release_cl(tc::mapa(&ifull[slot], 0));
        tc::mbar_arrive_release_cl(tc::mapa(&ifull[slot], 1));
        if (item < 0) break;
      }
      // the last scheduler to finish leaves the counters zero for the next launch
      if (a.sched && atomicAdd(&a.sched[1], 1) == nclusters - 1) {
        a.sched[0] = 0;
        a.sched[1] = 0;
      }
    } else if (warp == 2 && lane == 0 && rank == 0) {
      // ------------------------------------------------------------ MMA issuer (rank 0)
      int use = 0, j = 0;
      bool ok = true;
      for (int iu = 0; ok; ++iu) {
        const int item = tc_ring_item(iu, ifull, iring, iempty, a.status);
        if (item < 0) {
          ok = item == -1;
          break;
        }
        int e, p, m0, rows, n;
        tc_decode_item(item, tprefix, a.num_e, soff, tdesc, e, p, m0, rows, n);
        const uint32_t idesc = tc::idesc_bf16_m256((uint32_t)n);
        for (int kb = 0; kb < nkb && ok; ++kb, ++j) {
          const int slot = j & 1;
          if (!tc::mbar_spin_cl(&pempty[slot], ((j >> 1) & 1) ^ 1, a.status)) {
            ok = false;
            break;
          }
          tc::fence_after_sync();
          for (int h = 0; h < 2; ++h, ++use) {
            const int sa = use % SA;
            if (!tc::mbar_spin_cl(&abfull[sa], (use / SA) & 1, a.status)) {
              ok = false;
              break;
            }
            tc::fence_after_sync();
            const uint32_t abase = smem_u32(ab + sa * C::kAB);
#pragma unroll
            for (int ks = 0; ks < 4; ++ks)
              tc::mma_ss2(tmem + slot * 256, tc::sdesc_sw128(abase + ks * 32), tc::sdesc_sw128(abase + 16384 + ks * 32),
                          idesc, (h | ks) != 0);
            tc::commit2_mc(&abempty[sa], 3);
          }
          if (ok) tc::commit2_mc(&pfull[slot], 3);
        }
      }
      tc::commit2_mc(drain, 1);  // all MMAs issued above have completed once this lands
      mbar_wait(drain, 0, a.status);
    }
  } else if (warp < 12) {
    // ------------------------------------------------------------ dequant warpgroups
    tc::setmaxnreg_dec<kRegDequant>();
    const int dq = (warp - 4) * 32 + lane;
    const int r = dq & 127, hk = dq >> 7;  // weight row and 32-k half of the stage of this thread
    int use = 0;
    bool ok = true;
    for (int iu = 0; ok; ++iu) {
      const int item = tc_ring_item_warp(iu, ifull, iring, iempty, a.status, lane);
      if (item < 0) {
        ok = item == -1;
        break;
      }
      int e, p, m0, rows, n;
      tc_decode_item(item, tprefix, a.num_e, soff, tdesc, e, p, m0, rows, n);
      const bool valid = 2 * p + (int)rank < ntiles;
      for (int st = 0; st < nstages; ++st, ++use) {
        const int s = use % SW, sa = use % SA;
        const bool got = mbar_wait(&wfull[s], (use / SW) & 1, a.status) &&
                         tc::mbar_wait_cl(&abempty[sa], ((use / SA) & 1) ^ 1, a.status);
        if (!__all_sync(0xffffffffu, got)) {  // the warp leaves together (it shares collectives)
          ok = false;
          break;
        }
        if (valid) {
          const uint8_t* half = wtiles + s * C::kWBytes;
          dequant_half_row<FMT>(half, half + C::kHalfW + (BK::kZeros ? 256 : 0), r, hk, ab + sa * C::kAB);
        }
        tc::fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&wempty[s]);
          tc::mbar_arrive_cl(tc::mapa(&abfull[sa], 0));
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue warpgroups
    tc::setmaxnreg_inc<kRegEpilogue>();
    const int ewg = (warp - 12) >> 2;  // token columns [128 ewg, 128 ewg + 128)
    const int q = warp & 3;           // tensor-memory lane quarter
    const int r = q * 32 + lane;      // weight row of this thread
    const uint32_t tl = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(ewg * 128);
    float* xb = xchg + ewg * 128 * C::kXRow;
    float* wsm = reinterpret_cast<float*>(smem + C::kRowWOff) + ewg * 128;  // FFN2: weights of the WG's tokens
    int ffn1_use = 0;  // FFN1: output chunks staged so far (buffer = ffn1_use & 1)
    const uint32_t pe0 = tc::mapa(&pempty[0], 0), pe1 = tc::mapa(&pempty[1], 0);
    int j = 0;
    bool ok = true;
    for (int iu = 0; ok; ++iu) {
      const int item = tc_ring_item_warp(iu, ifull, iring, iempty, a.status, lane);
      if (item < 0) {
        ok = item == -1;
        break;
      }
      int e, p, m0, rows, n;
      tc_decode_item(item, tprefix, a.num_e, soff, tdesc, e, p, m0, rows, n);
      const int blk = 2 * p + (int)rank;
      const bool valid = blk < ntiles;
      const int ncols = max(0, min(128, n - ewg * 128));
      const uint8_t* wb = a.w + (size_t)e * a.expert_stride + (size_t)(valid ? blk : 0) * ktiles * BK::kBytes;
      const int row0 = soff[e] + m0;
      // FFN2: this thread's token's routing weight, loaded now so that its latency passes
      // under the item's k loop (staged through shared memory for the output phase)
      float my_wr = 1.f;
      if constexpr (MODE == kFfn2)
        if (valid && a.row_weight && ewg * 128 + r < rows) my_wr = __ldg(a.row_weight + row0 + ewg * 128 + r);
      float tot[128];
#pragma unroll
      for (int i = 0; i < 128; ++i) tot[i] = 0.f;
      // scales of k-blocks kb and kb + 1 in flight while kb is promoted (their loads are
      // issued two blocks ahead, so the global-load latency stays off the promotion path)
      float s_cur = valid ? block_scale<FMT, MODE>(wb, r) : 0.f;
      float s_nxt = (valid && nkb > 1) ? block_scale<FMT, MODE>(wb + BK::kBytes, r) : 0.f;
      for (int kb = 0; kb < nkb; ++kb, ++j) {
        const int slot = j & 1;
        const float s = s_cur;
        s_cur = s_nxt;
        s_nxt = (valid && kb + 2 < nkb) ? block_scale<FMT, MODE>(wb + (size_t)(kb + 2) * BK::kBytes, r) : 0.f;
        if (!__all_sync(0xffffffffu, tc::mbar_wait_cl(&pfull[slot], (j >> 1) & 1, a.status))) {
          ok = false;  // the warp leaves together (tensor-memory loads are warp-wide)
          break;
        }
        tc::fence_after_sync();
#pragma unroll
        for (int c = 0; c < 128; c += 32) {
          if (c < ncols) {  // uniform over the warpgroup
            uint32_t v[32];  // 32 columns per load (ncols is a multiple of 32)
            tc::ld_32x32b_x32(tl + (uint32_t)(slot * 256 + c), v);
            tc::wait_ld();
            promote16(tot + c, *reinterpret_cast<const uint32_t(*)[16]>(v), s);
            promote16(tot + c + 16, *reinterpret_cast<const uint32_t(*)[16]>(v + 16), s);
          }
        }
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive_cl(slot ? pe1 : pe0);
      }
      if (!ok || !valid) continue;
      // Output, 16 tokens at a time.  FFN2: bf16 rows are staged token-major in shared memory
      // and each warp writes whole token rows, lane l channels 4l .. 4l + 3; fp32 rows go
      // straight from the registers.  FFN1: see below.
      if constexpr (MODE == kFfn2) {
        wsm[r] = my_wr;  // read after the first chunk's barrier
#pragma unroll
      for (int c = 0; c < 128; c += 16) {
        if (c < ncols) {  // uniform over the warpgroup
          {
            if (a.out_bf16) {  // uniform: staged token-major, each warp writes 4 tokens' 256-byte rows
#pragma unroll
              for (int i = 0; i < 16; ++i) xb[i * C::kTokPitch + r] = tot[c + i];
              named_bar(1 + ewg, 128);
              // the warp's 4 tokens: all shared-memory reads first, then the 4 row stores
              float4 v4[4];
              float wr4[4];
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                v4[j] = *reinterpret_cast<const float4*>(xb + (q * 4 + j) * C::kTokPitch + 4 * lane);
                wr4[j] = wsm[c + q * 4 + j];
              }
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                const int tl = q * 4 + j;  // token of the chunk (uniform over the warp)
                if (ewg * 128 + c + tl < rows) {
                  const __nv_bfloat162 h0 = __floats2bfloat162_rn(v4[j].x * wr4[j], v4[j].y * wr4[j]);
                  const __nv_bfloat162 h1 = __floats2bfloat162_rn(v4[j].z * wr4[j], v4[j].w * wr4[j]);
                  uint16_t* orow = static_cast<uint16_t*>(a.out) + (size_t)(row0 + ewg * 128 + c + tl) * a.out_ld +
                                   blk * kTileN + 4 * lane;
                  *reinterpret_cast<uint2*>(orow) =
                      make_uint2(*reinterpret_cast<const uint32_t*>(&h0), *reinterpret_cast<const uint32_t*>(&h1));
                }
              }
              named_bar(1 + ewg, 128);
              continue;
            }
            // fp32 straight from the registers: for each token the warp's 32 lanes hold 32
            // consecutive channels, so one 4-byte store per lane writes a whole 128-byte line
            if (c == 0) named_bar(1 + ewg, 128);  // the item's routing weights are staged
            float* orow = static_cast<float*>(a.out) + (size_t)(row0 + ewg * 128 + c) * a.out_ld + blk * kTileN + r;
#pragma unroll
            for (int i = 0; i < 16; i += 4) {
              const float4 wr = *reinterpret_cast<const float4*>(wsm + c + i);
              const float w4[4] = {wr.x, wr.y, wr.z, wr.w};
#pragma unroll
              for (int u = 0; u < 4; ++u)
                if (ewg * 128 + c + i + u < rows) orow[(size_t)(i + u) * a.out_ld] = tot[c + i + u] * w4[u];
            }
            if (c + 16 >= ncols) named_bar(1 + ewg, 128);  // weights read before the next item's
          }
        }
      }
      } else {
#pragma unroll
      for (int c = 0; c < 64; c += 16) {
        if (c < ncols) {  // uniform over the warpgroup
          {
            // rows 2i / 2i + 1 hold the gate / up sums of channel i (i = r >> 1) in adjacent
            // lanes: a shuffle gives the even lane the up sums of tokens c .. c + 15 and the odd
            // lane the gate sums of tokens 64 + c .. 64 + c + 15, so the even lane writes
            // SwiGLU for the first and the odd lane for the second 16 tokens of the chunk,
            // staged as bf16 token rows (two buffers, one barrier per chunk) and stored as
            // 16-byte vectors, four whole 128-byte rows per warp instruction.
            const bool up_row = r & 1;
            uint16_t* buf = reinterpret_cast<uint16_t*>(xb) + (ffn1_use & 1) * C::kFfn1Buf;
            uint16_t* mine = buf + (up_row ? C::kFfn1Odd : 0) + (r >> 1);
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const float other = __shfl_xor_sync(0xffffffffu, up_row ? tot[c + i] : tot[64 + c + i], 1);
              const float g = up_row ? other : tot[c + i];
              const float u = up_row ? tot[64 + c + i] : other;
              mine[i * 64] = __bfloat16_as_ushort(__float2bfloat16_rn(__fdividef(g, 1.0f + __expf(-g)) * u));
            }
            named_bar(1 + ewg, 128);
            const int wt = r >> 3, part = r & 7;  // 16 tokens of each half: 8 x 16-byte parts per token row
#pragma unroll
            for (int pass = 0; pass < 2; ++pass) {
              const int tl = wt + 16 * pass;  // 0..15: tokens c + tl; 16..31: tokens 64 + c + tl - 16
              const int tok = ewg * 128 + (pass == 0 ? c + tl : 64 + c + tl - 16);
              if (tok < rows) {
                const uint4 v =
                    *reinterpret_cast<const uint4*>(buf + (pass ? C::kFfn1Odd + (tl - 16) * 64 : tl * 64) + part * 8);
                *reinterpret_cast<uint4*>(static_cast<uint16_t*>(a.out) + (size_t)(row0 + tok) * a.out_ld + blk * 64 +
                                          part * 8) = v;
              }
            }
            ++ffn1_use;
          }
        }
      }
      }
    }
  }

  tc::fence_before_sync();
  __syncthreads();
  tc::cluster_sync();  // no MMA, remote arrival or tensor-memory read of either CTA is in flight
  if (warp == 2) {
    tc::fence_after_sync();
    tc::tmem_dealloc2(tmem, 512);
  }
}

// Clusters of two that fit the device at once (one CTA per SM), per device.
template <int FMT, int MODE>
static int tc_clusters(int num_sms) {
  static std::atomic<int> cache[64];
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  if (dev >= 0 && dev < 64) {
    const int c = cache[dev].load(std::memory_order_relaxed);
    if (c > 0) return c;
  }
  using C = TcCfg<FMT>;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(num_sms / 2 * 2);
  cfg.blockDim = dim3(C::kThreads);
  cfg.dynamicSmemBytes = C::kSmem;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, tc_gemm_kernel<FMT, MODE>, &cfg) != cudaSuccess || n < 1) n = num_sms / 2;
  if (dev >= 0 && dev < 64) cache[dev].store(n, std::memory_order_relaxed);
  return n;
}

template <int FMT, int MODE>
static int launch_tc_t(const CUtensorMap& map, const TcArgs& a, int num_sms, cudaStream_t st) {
  using C = TcCfg<FMT>;
  auto kern = tc_gemm_kernel<FMT, MODE>;
  static std::atomic<uint64_t> smem_set{0};  // devices with the shared-memory limit raised
  const int rc = ensure_smem_limit(kern, C::kSmem, smem_set);
  if (rc) return rc;
  const int nc = tc_clusters<FMT, MODE>(num_sms);
  if (nc < 1) return CCUT_ERR_CUDA;
  return launch_k(kern, dim3(2 * nc), dim3(C::kThreads), C::kSmem, st, map, a);
}

int launch_tc_gemm(int fmt, int mode, const CUtensorMap& map, const TcArgs& a, int num_sms, cudaStream_t st) {
  switch (fmt) {
    case CCUT_FMT_AWQ_INT4_G128:
      return mode == kFfn1 ? launch_tc_t<CCUT_FMT_AWQ_INT4_G128, kFfn1>(map, a, num_sms, st)
                           : launch_tc_t<CCUT_FMT_AWQ_INT4_G128, kFfn2>(map, a, num_sms, st);
    case CCUT_FMT_INT4_SYM_G128:
      return mode == kFfn1 ? launch_tc_t<CCUT_FMT_INT4_SYM_G128, kFfn1>(map, a, num_sms, st)
                           : launch_tc_t<CCUT_FMT_INT4_SYM_G128, kFfn2>(map, a, num_sms, st);
    case CCUT_FMT_FP8_E4M3_CH:
      return mode == kFfn1 ? launch_tc_t<CCUT_FMT_FP8_E4M3_CH, kFfn1>(map, a, num_sms, st)
                           : launch_tc_t<CCUT_FMT_FP8_E4M3_CH, kFfn2>(map, a, num_sms, st);
    default:
      return mode == kFfn1 ? launch_tc_t<CCUT_FMT_FP8_E4M3_B128, kFfn1>(map, a, num_sms, st)
                           : launch_tc_t<CCUT_FMT_FP8_E4M3_B128, kFfn2>(map, a, num_sms, st);
  }
}

}  // namespace ccut
