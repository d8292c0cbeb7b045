// tc_gemm.cu -- tcgen05 dequant-fused grouped expert GEMM (gate/up + SiLU, and down).
//
// Swap-AB formulation: the 128 output channels of a weight tile are the MMA's M dimension
// (A operand, in tensor memory), the NT tokens of a row tile are N (B operand, in shared
// memory), and the fp32 accumulators live in tensor memory:
//   D[channel, token] (+)= A[channel, k] * B[token, k]      (tcgen05.mma kind::f16, M=128)
//
// Work item = (expert, token tile of NT rows, 128-channel tile); one persistent CTA per SM
// walks the items.  Warp roles inside the CTA (24 warps):
//   warp 0        producer: per 128-k stage one bulk copy of the packed weight block(s)
//                 and two 128-byte-swizzled TMA tile loads of the activation rows
//   warp 1        MMA issuer (one thread) and tensor-memory owner
//   warp 2        builds the item prefix, then idles
//   warps 4..19   four dequant warpgroups: each thread owns one weight row (channel) and
//                 converts a k-slice of it to f16 with the group/block scale applied
//                 ((q - z) * s for AWQ, e4m3 * S for FP8), storing it to tensor memory as
//                 the A operand of the next MMAs (gate/up: warpgroup g converts matrix g/2,
//                 k half g%2; down: k quarter g)
//   warps 20..23  epilogue warpgroup: tensor memory -> registers -> silu(gate) * up as
//                 f16 rows (gate/up), or row_weight * acc as fp32 rows (down)
// Stages are guarded by mbarriers (full: copies landed; empty: dequant done reading and
// the MMAs that read the activations completed); A buffers and accumulators are
// double-buffered through their own mbarrier pairs.  Every wait is bounded.
//
// Follows ccut/blocks/moe.py:122-141 (expert_ffn), ccut/quant/kernels.py:219-231 (SiLU),
// the dequant of ccut/quant/kernels.py:150-171 / :276-295 (restated for the group-128 /
// block-128 formats) and ccut/models/generic.py:377-378 (routing-weight scaling).
#include "kernels.cuh"
#include "tc.cuh"

namespace ccut {

// Debug-only per-CTA cycle counters of the role waits (built only with -DCCUT_TC_PROFILE).
#ifdef CCUT_TC_PROFILE
__device__ unsigned long long g_tc_prof[1024][12];
#define TC_PROF_START(v) const long long v = clock64()
#define TC_PROF_ADD(slot, v) atomicAdd(&g_tc_prof[blockIdx.x & 1023][slot], (unsigned long long)(clock64() - (v)))
#else
#define TC_PROF_START(v)
#define TC_PROF_ADD(slot, v)
#endif

template <int FMT, int MODE, int NT>
struct TcCfg {
  static constexpr int kNMat = MODE == kFfn1 ? 2 : 1;
  static constexpr int kBlk = Blk<FMT>::kBytes;
  static constexpr int kWBytes = kNMat * kBlk;
  static constexpr int kWPad = (kWBytes + 1023) / 1024 * 1024;
  static constexpr int kBBytes = 2 * NT * 128;  // two 64-k boxes of NT rows x 128 B
  static constexpr int kStageBytes = kWPad + kBBytes;
  static constexpr int kStages0 = (200 * 1024) / kStageBytes;
  static constexpr int kStages = kStages0 > 8 ? 8 : kStages0;
  // Tensor memory (512 columns): accumulators D [kND x kNMat x NT] first, then a ring of
  // kNA A-operand buffers [kNMat x 64 columns] (one 128-k stage of f16 weights).
  static constexpr int kND = (2 * kNMat * NT + kNMat * 128 <= 512) ? 2 : 1;  // accumulator buffers
  static constexpr int kDCols = kND * kNMat * NT;
  static constexpr int kNA0 = (512 - kDCols) / (kNMat * 64);
  static constexpr int kNA = kNA0 > 4 ? 4 : kNA0;  // A-operand buffers
  static constexpr int kThreads = 768;
  static constexpr int kDeqWarps = 16;
  static constexpr int kNBar = 2 * kStages + 2 * 4 + 2 * 2 + 1;
  static constexpr int kHeader = kNBar * 8 + 16 + 4 * (kMaxExperts + 1);
  static constexpr int kHeaderAligned = (kHeader + 1023) / 1024 * 1024;
  static constexpr int kSmem = kHeaderAligned + kStages * kStageBytes + 1024;  // +1024: runtime alignment slack
  static_assert(kStages >= 2, "stage does not fit");
  static_assert(NT % 16 == 0 && NT >= 16 && NT <= 128, "token tile must be 16..128, multiple of 16");
  static_assert(kNA >= 2 && kDCols + kNA * kNMat * 64 <= 512, "tensor-memory budget");
  static_assert(kSmem <= 227 * 1024, "shared memory budget");
};

template <class C, int NT>
__device__ __forceinline__ uint32_t dcol(int db, int m) { return (uint32_t)((db * C::kNMat + m) * NT); }
template <class C>
__device__ __forceinline__ uint32_t acol(int a, int m) { return (uint32_t)(C::kDCols + (a * C::kNMat + m) * 64); }

template <int NT>
__device__ __forceinline__ void tc_decode_item(int item, const int* tprefix, int num_e, const int* offsets,
                                               int& e, int& nt, int& m0, int& rows) {
  int lo = 0, hi = num_e - 1;  // last e with tprefix[e] <= item
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (tprefix[mid] <= item) lo = mid;
    else hi = mid - 1;
  }
  e = lo;
  const int me = offsets[e + 1] - offsets[e];
  const int mtiles = (me + NT - 1) / NT;
  const int local = item - tprefix[e];
  nt = local / mtiles;
  const int mt = local % mtiles;
  m0 = mt * NT;
  rows = min(NT, me - m0);
}

// f16x2 helpers
__device__ __forceinline__ uint32_t h2_sub(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t h2_mul(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t nib2_f16_1024(uint32_t w) {  // (1024 + q_lo, 1024 + q_hi)
  uint32_t v;
  asm("lop3.b32 %0, %1, 0x000F000F, 0x64006400, 0xEA;" : "=r"(v) : "r"(w));
  return v;
}

// Dequantize k in [kbase, kbase + 2*NREG) of row r of a row-layout block into NREG f16x2
// registers (register i = k kbase+2i, kbase+2i+1); kbase is a multiple of 32.
template <int FMT, int NREG>
__device__ __forceinline__ void dequant_slice(const uint8_t* blk, int r, int kbase, uint32_t zz, uint32_t ss,
                                              uint32_t (&v)[NREG]) {
  if constexpr (FMT == CCUT_FMT_FP8_E4M3_B128) {
#pragma unroll
    for (int c = 0; c < NREG / 8; ++c) {  // 16-byte chunks of 16 e4m3 values
      const int cc = kbase / 16 + c;
      const uint4 q = *reinterpret_cast<const uint4*>(blk + r * 128 + 16 * (cc ^ (r & 7)));
      const uint32_t w4[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
      for (int p = 0; p < 8; ++p)
        v[c * 8 + p] = h2_mul(e4m3x2_to_f16x2(static_cast<uint16_t>(w4[p >> 1] >> (16 * (p & 1)))), ss);
    }
  } else {
#pragma unroll
    for (int c = 0; c < NREG / 16; ++c) {  // 16-byte chunks of 32 nibbles
      const int cc = kbase / 32 + c;
      const uint4 q = *reinterpret_cast<const uint4*>(blk + r * 64 + 16 * (cc ^ ((r >> 1) & 3)));
      const uint32_t w4[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int i = 0; i < 4; ++i)
          v[(c * 4 + j) * 4 + i] = h2_mul(h2_sub(nib2_f16_1024(w4[j] >> (4 * i)), zz), ss);
    }
  }
}

template <int FMT, int MODE, int NT>
__global__ void __launch_bounds__(768, 1) tc_gemm_kernel(const __grid_constant__ CUtensorMap bmap, TcArgs a) {
  using C = TcCfg<FMT, MODE, NT>;
  using BK = Blk<FMT>;
  constexpr int S = C::kStages;
  constexpr int NM = C::kNMat;
  constexpr int ND = C::kND;
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte alignment for the 128-byte-swizzled operand tiles
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem);
  uint64_t* full = bars;
  uint64_t* empty = bars + S;
  uint64_t* afull = bars + 2 * S;
  uint64_t* aempty = afull + 4;
  uint64_t* dfull = aempty + 4;
  uint64_t* dempty = dfull + 2;
  uint64_t* drain = dempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + C::kNBar);
  int* tprefix = reinterpret_cast<int*>(smem + C::kNBar * 8 + 16);
  uint8_t* stages = smem + C::kHeaderAligned;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ntiles = a.N / kTileN, ktiles = a.K / kTileK;
  TC_PROF_START(t_kernel);

  if (warp == 1) {
    tc::tmem_alloc(tmem_slot, 512);
    tc::tmem_relinquish();
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], C::kDeqWarps + 1);
    }
    for (int i = 0; i < 4; ++i) {
      mbar_init(&afull[i], C::kDeqWarps);
      mbar_init(&aempty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&dfull[i], 1);
      mbar_init(&dempty[i], 4);
    }
    mbar_init(drain, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    tc::prefetch_tmap(&bmap);
  }
  if (warp == 2) {  // item prefix over experts: tiles(e) = ceil(M_e / NT) * ntiles
    int carry = 0;
    for (int b = 0; b < a.num_e; b += 32) {
      const int e = b + lane;
      const int me = e < a.num_e ? a.offsets[e + 1] - a.offsets[e] : 0;
      const int c = ((me + NT - 1) / NT) * ntiles;
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
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  const int total = tprefix[a.num_e];

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int use = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < total && ok; item += gridDim.x) {
        int e, nt, m0, rows;
        tc_decode_item<NT>(item, tprefix, a.num_e, a.offsets, e, nt, m0, rows);
        const int row0 = a.offsets[e] + m0;
        const uint8_t* wb = a.w + (size_t)e * a.expert_stride + (size_t)nt * ktiles * C::kWBytes;
        for (int kt = 0; kt < ktiles; ++kt, ++use) {
          const int s = use % S;
          TC_PROF_START(p0);
          if (!mbar_wait(&empty[s], ((use / S) & 1) ^ 1, a.status)) {
            ok = false;
            break;
          }
          TC_PROF_ADD(0, p0);
          uint8_t* st = stages + s * C::kStageBytes;
          mbar_arrive_expect_tx(&full[s], C::kWBytes + C::kBBytes);
          bulk_g2s(st, wb + (size_t)kt * C::kWBytes, C::kWBytes, &full[s]);
          tc::tma_load_2d(st + C::kWPad, &bmap, kt * kTileK, row0, &full[s]);
          tc::tma_load_2d(st + C::kWPad + NT * 128, &bmap, kt * kTileK + 64, row0, &full[s]);
        }
      }
      if (!ok)  // let issued copies land before the CTA exits
        for (int u = use > S ? use - S : 0; u < use; ++u) mbar_wait(&full[u % S], (u / S) & 1, nullptr);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = tc::idesc_f16_m128(NT);
      int use = 0, it = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < total && ok; item += gridDim.x, ++it) {
        const int db = it % ND;
        TC_PROF_START(m0);
        if (!mbar_wait(&dempty[db], ((it / ND) & 1) ^ 1, a.status)) break;
        TC_PROF_ADD(3, m0);
        tc::fence_after_sync();
        for (int kt = 0; kt < ktiles; ++kt, ++use) {
          const int s = use % S, ab = use % C::kNA;
          TC_PROF_START(m1);
          const bool okf = mbar_wait(&full[s], (use / S) & 1, a.status);
          TC_PROF_ADD(1, m1);
          TC_PROF_START(m2);
          if (!okf || !mbar_wait(&afull[ab], (use / C::kNA) & 1, a.status)) {
            ok = false;
            break;
          }
          TC_PROF_ADD(2, m2);
          tc::fence_after_sync();
          const uint32_t bbase = smem_u32(stages + s * C::kStageBytes + C::kWPad);
#pragma unroll
          for (int m = 0; m < NM; ++m)
#pragma unroll
            for (int ks = 0; ks < 8; ++ks) {
              const uint64_t bd = tc::sdesc_sw128(bbase + (ks >> 2) * (NT * 128) + (ks & 3) * 32);
              tc::mma_ts(tmem + dcol<C, NT>(db, m), tmem + acol<C>(ab, m) + ks * 8, bd, idesc, (kt | ks) != 0);
            }
          tc::commit(&aempty[ab]);
          tc::commit(&empty[s]);
        }
        if (ok) tc::commit(&dfull[db]);
      }
      tc::commit(drain);  // all MMAs issued above have completed once this lands
      mbar_wait(drain, 0, a.status);
    }
  } else if (warp >= 4 && warp < 20) {
    // ------------------------------------------------------------ dequant warpgroups
    const int wg = (warp - 4) >> 2;
    const int q = warp & 3;       // tensor-memory lane quarter
    const int r = q * 32 + lane;  // weight row (output channel) of this thread
    const int mat = NM == 2 ? (wg >> 1) : 0;
    constexpr int kSliceK = NM == 2 ? 64 : 32;  // k handled per warpgroup and stage
    const int kbase = NM == 2 ? 64 * (wg & 1) : 32 * wg;
    const uint32_t tlane = (uint32_t)(q * 32) << 16;
    int use = 0;
    bool ok = true;
    for (int item = blockIdx.x; item < total && ok; item += gridDim.x) {
      for (int kt = 0; kt < ktiles; ++kt, ++use) {
        const int s = use % S, ab = use % C::kNA;
        const bool rec = (warp == 4 && lane == 0);
        (void)rec;
        TC_PROF_START(d0);
        const bool okf = mbar_wait(&full[s], (use / S) & 1, a.status);
        if (rec) TC_PROF_ADD(4, d0);
        TC_PROF_START(d1);
        if (!okf || !mbar_wait(&aempty[ab], ((use / C::kNA) & 1) ^ 1, a.status)) {
          ok = false;
          break;
        }
        if (rec) TC_PROF_ADD(5, d1);
        TC_PROF_START(d2);
        tc::fence_after_sync();
        const uint8_t* blk = stages + s * C::kStageBytes + mat * C::kBlk;
        uint32_t zz = 0, ss;
        if constexpr (FMT == CCUT_FMT_AWQ_INT4_G128) {
          const uint32_t z = (blk[BK::kZeroOff + (r >> 1)] >> (4 * (r & 1))) & 0xF;
          zz = (0x6400u | z) * 0x10001u;
          const uint32_t sh = reinterpret_cast<const uint16_t*>(blk + BK::kScaleOff)[r];
          ss = sh * 0x10001u;
        } else {
          const __half2 s2 = __float2half2_rn(reinterpret_cast<const float*>(blk + BK::kScaleOff)[0]);
          ss = *reinterpret_cast<const uint32_t*>(&s2);
        }
        const uint32_t taddr = tmem + tlane + acol<C>(ab, mat) + kbase / 2;
        if constexpr (kSliceK == 64) {
          uint32_t v[32];
          dequant_slice<FMT, 32>(blk, r, kbase, zz, ss, v);
          tc::st_32x32b_x32(taddr, v);
        } else {
          uint32_t v[16];
          dequant_slice<FMT, 16>(blk, r, kbase, zz, ss, v);
          tc::st_32x32b_x16(taddr, v);
        }
        if (rec) TC_PROF_ADD(6, d2);
        TC_PROF_START(d3);
        tc::wait_st();
        if (rec) TC_PROF_ADD(10, d3);
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&afull[ab]);
          mbar_arrive(&empty[s]);
        }
      }
    }
  } else if (warp >= 20) {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;
    const int c = q * 32 + lane;  // channel within the 128-tile
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    int it = 0;
    for (int item = blockIdx.x; item < total; item += gridDim.x, ++it) {
      const int db = it % ND;
      // item metadata and routing weights first: their latency overlaps the MMAs
      int e, nt, m0, rows;
      tc_decode_item<NT>(item, tprefix, a.num_e, a.offsets, e, nt, m0, rows);
      const int row0 = a.offsets[e] + m0;
      float wl[NT / 32];  // routing weight of token 32*i + lane
#pragma unroll
      for (int i = 0; i < NT / 32; ++i) {
        const int tok = 32 * i + lane;
        wl[i] = (MODE == kFfn2 && a.row_weight && tok < rows) ? a.row_weight[row0 + tok] : 1.f;
      }
      TC_PROF_START(e0);
      if (!mbar_wait(&dfull[db], (it / ND) & 1, a.status)) break;
      if (warp == 20 && lane == 0) TC_PROF_ADD(7, e0);
      TC_PROF_START(e1);
      tc::fence_after_sync();
      const int n = nt * kTileN + c;
#pragma unroll
      for (int c0 = 0; c0 < NT; c0 += 16) {
        if (c0 < rows) {
          if constexpr (MODE == kFfn1) {
            uint32_t g[16], u[16];
            tc::ld_32x32b_x16(tmem + lane_base + dcol<C, NT>(db, 0) + c0, g);
            tc::ld_32x32b_x16(tmem + lane_base + dcol<C, NT>(db, 1) + c0, u);
            tc::wait_ld();
            uint16_t* orow = static_cast<uint16_t*>(a.out) + (size_t)(row0 + c0) * a.out_ld + n;
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              if (c0 + j < rows) {
                const float gv = __uint_as_float(g[j]);
                const float hv = __fdividef(gv, 1.0f + __expf(-gv)) * __uint_as_float(u[j]);
                orow[(size_t)j * a.out_ld] = __half_as_ushort(__float2half_rn(hv));
              }
            }
          } else {
            uint32_t d[16];
            tc::ld_32x32b_x16(tmem + lane_base + dcol<C, NT>(db, 0) + c0, d);
            tc::wait_ld();
            float* orow = static_cast<float*>(a.out) + (size_t)(row0 + c0) * a.out_ld + n;
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const float wr = __shfl_sync(0xffffffffu, wl[(c0 + j) / 32], (c0 + j) % 32);
              if (c0 + j < rows) orow[(size_t)j * a.out_ld] = __uint_as_float(d[j]) * wr;
            }
          }
        }
      }
      tc::fence_before_sync();
      __syncwarp();
      if (warp == 20 && lane == 0) TC_PROF_ADD(8, e1);
      if (lane == 0) mbar_arrive(&dempty[db]);
    }
  }

  tc::fence_before_sync();
  __syncthreads();
  if (threadIdx.x == 0) TC_PROF_ADD(9, t_kernel);
  if (warp == 1) {
    __syncwarp();
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, 512);
  }
}

template <int FMT, int MODE, int NT>
static int launch_tc_t(const CUtensorMap& map, const TcArgs& a, int num_sms, cudaStream_t st) {
  using C = TcCfg<FMT, MODE, NT>;
  auto kern = tc_gemm_kernel<FMT, MODE, NT>;
  static int attr_done = -1;  // device the attribute was set for
  int dev = 0;
  cudaGetDevice(&dev);
  if (attr_done != dev) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmem) != cudaSuccess)
      return CCUT_ERR_CUDA;
    attr_done = dev;
  }
  kern<<<num_sms, C::kThreads, C::kSmem, st>>>(map, a);
  return cudaPeekAtLastError() == cudaSuccess ? CCUT_OK : CCUT_ERR_CUDA;
}

template <int MODE, int NT>
static int launch_tc_fmt(int fmt, const CUtensorMap& map, const TcArgs& a, int num_sms, cudaStream_t st) {
  if (fmt == CCUT_FMT_AWQ_INT4_G128) return launch_tc_t<CCUT_FMT_AWQ_INT4_G128, MODE, NT>(map, a, num_sms, st);
  return launch_tc_t<CCUT_FMT_FP8_E4M3_B128, MODE, NT>(map, a, num_sms, st);
}

#ifdef CCUT_TC_PROFILE
extern "C" __attribute__((visibility("default"))) int ccut_debug_tc_prof(unsigned long long* host, int clear) {
  if (cudaMemcpyFromSymbol(host, g_tc_prof, sizeof(g_tc_prof)) != cudaSuccess) return CCUT_ERR_CUDA;
  if (clear) {
    static unsigned long long zeros[1024][12];
    if (cudaMemcpyToSymbol(g_tc_prof, zeros, sizeof(zeros)) != cudaSuccess) return CCUT_ERR_CUDA;
  }
  return CCUT_OK;
}
#endif

int tc_token_tile(int rows_per_expert) { return rows_per_expert <= 16 ? 32 : rows_per_expert <= 48 ? 64 : 128; }

int launch_tc_gemm(int fmt, int mode, int nt_tokens, const CUtensorMap& map, const TcArgs& a, int num_sms,
                   cudaStream_t st) {
  if (mode == kFfn1) {
    if (nt_tokens == 32) return launch_tc_fmt<kFfn1, 32>(fmt, map, a, num_sms, st);
    if (nt_tokens == 64) return launch_tc_fmt<kFfn1, 64>(fmt, map, a, num_sms, st);
    return launch_tc_fmt<kFfn1, 128>(fmt, map, a, num_sms, st);
  }
  if (nt_tokens == 32) return launch_tc_fmt<kFfn2, 32>(fmt, map, a, num_sms, st);
  if (nt_tokens == 64) return launch_tc_fmt<kFfn2, 64>(fmt, map, a, num_sms, st);
  return launch_tc_fmt<kFfn2, 128>(fmt, map, a, num_sms, st);
}

}  // namespace ccut
