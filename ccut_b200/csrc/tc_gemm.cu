// tc_gemm.cu -- tcgen05 dequant-fused grouped expert GEMM (gate/up + SiLU, and down).
//
// Swap-AB formulation: the 128 rows of a weight tile are the MMA's M dimension (A operand,
// in tensor memory), the NT tokens of a row tile are N (B operand, in shared memory), and
// the fp32 accumulators live in tensor memory:
//   D[row, token] (+)= A[row, k] * B[token, k]      (tcgen05.mma kind::f16, M=128, K=16)
// A tcgen05.mma of M=128 occupies the tensor pipe for the same ~138 cycles at any N up to
// 256 (measured on B200), so full tensor throughput needs N = 256 token tiles.  Both the
// accumulators and a ring of A buffers must fit the 512 tensor-memory columns, so the gate
// and up matrices are fused into one A matrix (row tile t = 64 gate rows + the same 64 up
// rows) and a stage covers 64 k.
//
// Work item = (expert, token tile of NT rows, 128-row weight tile); one persistent CTA per
// SM walks the items.  Warp roles (28 warps):
//   warp 0        weight producer: per 64-k stage one bulk copy of the packed half block and
//                 one of its scale / zero-point metadata into the weight ring
//   warp 3        activation producer: per stage one 128-byte-swizzled TMA tile of the
//                 activation rows into the activation ring
//   warps 1, 2    MMA issuers (one thread each, one half of the token tile each); warp 1
//                 owns the tensor memory, warp 2 first builds the item prefix
//   warps 4..11   two dequant warpgroups: each thread owns one weight row and converts a 32-k
//                 slice of every stage to f16 with the group/block scale applied
//                 ((q - z) * s for AWQ, e4m3 * S for FP8), storing it to tensor memory as the
//                 A operand of the next MMAs
//   warps 12..27  four epilogue warpgroups (16-token chunk c goes to group c % 4): tensor
//                 memory -> registers -> silu(gate) * up as f16 rows (gate rows pair with up
//                 rows through shared memory), or row_weight * acc as fp32 rows (down); each
//                 warp loads its next chunk from tensor memory before storing the current one
// The weight ring has its own full/empty barriers (released by the dequant warps); a stage's
// A buffer and activation tile share one "ready" barrier (dequant arrivals plus the TMA's
// bytes) and one "done" barrier (one MMA commit per issuer), because every extra commit or
// wait in an MMA-issuing thread costs tensor throughput.  Accumulators have their own pair.
// Every wait is bounded.
//
// Follows ccut/blocks/moe.py:122-141 (expert_ffn), ccut/quant/kernels.py:219-231 (SiLU),
// the dequant of ccut/quant/kernels.py:150-171 / :276-295 (restated for the group-128 /
// block-128 formats) and ccut/models/generic.py:377-378 (routing-weight scaling).
#include <stdlib.h>

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
  using B = Blk<FMT>;
  static constexpr bool kAwq = FMT == CCUT_FMT_AWQ_INT4_G128;
  static constexpr int kHalfW = kAwq ? 4096 : 8192;  // weights of one 64-k half block
  static constexpr int kMeta = kAwq ? 320 : 16;      // scales + zero-points / block scale(s)
  static constexpr int kWBytes = kHalfW + kMeta;     // one weight stage (multiple of 16)
  static constexpr int kBBytes = NT * 128;           // one activation stage: 64 k x NT rows x 2 B
  // Two rings: weight stages (read by the dequant warps, released as soon as they are
  // converted) and activation stages (read by the MMAs, released on MMA completion), so the
  // HBM-latency weight loads can run further ahead than the activation tiles.
  static constexpr int kXRow = 20;  // floats per row of the SwiGLU exchange buffer (16 + pad)
  static constexpr int kXchg = 4 * 64 * kXRow * 4;
  static constexpr int kSW0 = (40 * 1024) / kWBytes;
  static constexpr int kSW = kSW0 > 8 ? 8 : kSW0;
  static constexpr int kSB0 = (220 * 1024 - 4096 - kXchg - kSW * kWBytes) / kBBytes;
  static constexpr int kSB = kSB0 > 8 ? 8 : kSB0;
  // tensor memory (512 columns): accumulators [kND x NT] then a ring of kNA A buffers of 32
  // columns (64 k of f16).  Double-buffered accumulators (epilogue overlapping the next
  // item) whenever a ring of at least four A buffers still fits.
  static constexpr int kND = (2 * NT + 4 * 32 <= 512) ? 2 : 1;
  static constexpr int kDCols = kND * NT;
  static constexpr int kNA0 = (512 - kDCols) / 32;
  static constexpr int kNA = kNA0 > 8 ? 8 : kNA0;
  // Stage u uses weight slot u % kSW, A buffer u % kNA and activation tile u % kSB; its
  // "ready" barrier (dequant arrivals + TMA bytes) and "done" barrier (one MMA commit) sit
  // in a ring of kL > max(kNA, kSB) slots, so each waiter can wait for "MMAs of stage
  // u - depth done" with its own depth.
  static constexpr int kL = 16;
  static constexpr int kDeqWarps = 8;
  static constexpr int kEpiWarps = 16;
  static constexpr int kEpiGroups = 4;
  static constexpr int kThreads = 28 * 32;
  static constexpr int kNBar = 2 * kL + 2 * kSW + 2 * 2 + 1;
  static constexpr int kHeader = kNBar * 8 + 16 + 4 * (kMaxExperts + 1);
  static constexpr int kHeaderAligned = (kHeader + 1023) / 1024 * 1024;
  static constexpr int kXchgOff = kHeaderAligned;
  static constexpr int kBOff = kXchgOff + (kXchg + 1023) / 1024 * 1024;  // 1024-aligned activation tiles
  static constexpr int kWOff = kBOff + kSB * kBBytes;
  static constexpr int kSmem = kWOff + kSW * kWBytes + 1024;  // +1024: runtime alignment slack
  static_assert(kSB >= 3 && kSW >= 4 && kL > kNA && kL > kSB, "rings do not fit");
  static_assert(NT % 64 == 0 && NT >= 64 && NT <= 256, "token tile must be 64, 128, 192 or 256");
  static_assert(kNA >= 2 && kDCols + kNA * 32 <= 512, "tensor-memory budget");
  static_assert(kSmem <= 227 * 1024, "shared memory budget");
};

template <class C>
__device__ __forceinline__ uint32_t acol(int a) { return (uint32_t)(C::kDCols + a * 32); }

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

// Dequantize k in [32 sub, 32 sub + 32) of row r of a staged half block into 16 f16x2
// registers (register i = k 32 sub + 2i, +1).
template <int FMT>
__device__ __forceinline__ void dequant_slice(const uint8_t* half, int r, int sub, uint32_t zz, uint32_t ss,
                                              uint32_t (&v)[16]) {
  if constexpr (FMT == CCUT_FMT_FP8_E4M3_B128) {
#pragma unroll
    for (int c2 = 0; c2 < 2; ++c2) {  // two 16-byte chunks of 16 e4m3 values
      const int c = 2 * sub + c2;
      const uint4 q = *reinterpret_cast<const uint4*>(half + r * 64 + 16 * (c ^ ((r >> 1) & 3)));
      const uint32_t w4[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
      for (int p = 0; p < 8; ++p)
        v[c2 * 8 + p] = h2_mul(e4m3x2_to_f16x2(static_cast<uint16_t>(w4[p >> 1] >> (16 * (p & 1)))), ss);
    }
  } else {
    const uint4 q = *reinterpret_cast<const uint4*>(half + r * 32 + 16 * (sub ^ ((r >> 2) & 1)));
    const uint32_t w4[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int i = 0; i < 4; ++i) v[j * 4 + i] = h2_mul(h2_sub(nib2_f16_1024(w4[j] >> (4 * i)), zz), ss);
  }
}

__device__ __forceinline__ void named_bar(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

template <int FMT, int MODE, int NT>
__global__ void __launch_bounds__(896, 1) tc_gemm_kernel(const __grid_constant__ CUtensorMap bmap, TcArgs a) {
  pdl_wait();
  pdl_trigger();
  using C = TcCfg<FMT, MODE, NT>;
  using BK = Blk<FMT>;
  constexpr int SB = C::kSB;
  constexpr int SW = C::kSW;
  constexpr int L = C::kL;
  constexpr int ND = C::kND;
  constexpr int NA = C::kNA;
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte alignment for the 128-byte-swizzled operand tiles
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem);
  uint64_t* sready = bars;       // [L] A converted + activation tile landed
  uint64_t* sdone = sready + L;  // [L] MMAs of the stage completed
  uint64_t* wfull = sdone + L;
  uint64_t* wempty = wfull + SW;
  uint64_t* dfull = wempty + SW;
  uint64_t* dempty = dfull + 2;
  uint64_t* drain = dempty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + C::kNBar);
  int* tprefix = reinterpret_cast<int*>(smem + C::kNBar * 8 + 16);
  float* xchg = reinterpret_cast<float*>(smem + C::kXchgOff);
  uint8_t* btiles = smem + C::kBOff;
  uint8_t* wtiles = smem + C::kWOff;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ntiles = a.N / kTileN, nstages = a.K / 64;
  TC_PROF_START(t_kernel);

  if (warp == 1) {
    tc::tmem_alloc(tmem_slot, 512);
    tc::tmem_relinquish();
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < L; ++s) {
      mbar_init(&sready[s], C::kDeqWarps + 1);
      mbar_init(&sdone[s], 2);
    }
    for (int s = 0; s < SW; ++s) {
      mbar_init(&wfull[s], 1);
      mbar_init(&wempty[s], C::kDeqWarps);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&dfull[i], 2);
      mbar_init(&dempty[i], C::kEpiWarps);
    }
    mbar_init(drain, 2);
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

  if (warp == 0 || warp == 3) {
    // ------------------------------------------------------------ producers
    // warp 0: weight stages (half block + metadata, bulk copies); warp 3: activation tiles (TMA)
    if (lane == 0) {
      const bool wprod = warp == 0;
      int use = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < total && ok; item += gridDim.x) {
        int e, nt, m0, rows;
        tc_decode_item<NT>(item, tprefix, a.num_e, a.offsets, e, nt, m0, rows);
        const int row0 = a.offsets[e] + m0;
        const uint8_t* wb = a.w + (size_t)e * a.expert_stride + (size_t)nt * (a.K / kTileK) * BK::kBytes;
        for (int st = 0; st < nstages; ++st, ++use) {
          TC_PROF_START(p0);
          if (wprod) {
            const int s = use % SW;
            if (!mbar_spin(&wempty[s], ((use / SW) & 1) ^ 1, a.status)) {
              ok = false;
              break;
            }
            TC_PROF_ADD(0, p0);
            uint8_t* sb = wtiles + s * C::kWBytes;
            const uint8_t* blk = wb + (size_t)(st >> 1) * BK::kBytes;
            mbar_arrive_expect_tx(&wfull[s], C::kWBytes);
            bulk_g2s(sb, blk + (st & 1) * C::kHalfW, C::kHalfW, &wfull[s]);
            bulk_g2s(sb + C::kHalfW, blk + BK::kScaleOff, C::kMeta, &wfull[s]);
          } else {
            // activation tile use % SB is free once the MMAs of stage use - SB completed
            const int v = use - SB;
            if (v >= 0 && !mbar_spin(&sdone[v % L], (v / L) & 1, a.status)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&sready[use % L], C::kBBytes);
            tc::tma_load_2d(btiles + (use % SB) * C::kBBytes, &bmap, st * 64, row0, &sready[use % L]);
          }
        }
      }
      if (!ok) {  // let issued copies land before the CTA exits
        const int R = wprod ? SW : SB;
        for (int u = use > R ? use - R : 0; u < use; ++u)
          mbar_wait(wprod ? &wfull[u % SW] : &sready[u % L], (u / (wprod ? SW : L)) & 1, nullptr);
      }
    }
  } else if (warp == 1 || warp == 2) {
    // ------------------------------------------------------------ MMA issuers
    // Two issuing threads, each driving the MMAs of one half of the token tile (a single
    // thread cannot issue tcgen05.mma fast enough to keep the tensor pipe busy).
    if (lane == 0) {
      const int half = warp - 1;
      const uint32_t idesc = tc::idesc_f16_m128(NT / 2);
      int use = 0, it = 0;
      bool ok = true;
      for (int item = blockIdx.x; item < total && ok; item += gridDim.x, ++it) {
        const int db = it % ND;
        TC_PROF_START(m0);
        if (!mbar_spin(&dempty[db], ((it / ND) & 1) ^ 1, a.status)) break;
        TC_PROF_ADD(3, m0);
        tc::fence_after_sync();
        for (int st = 0; st < nstages; ++st, ++use) {
          TC_PROF_START(m1);
          if (!mbar_spin(&sready[use % L], (use / L) & 1, a.status)) {
            ok = false;
            break;
          }
          TC_PROF_ADD(1, m1);
          TC_PROF_START(m3);
          tc::fence_after_sync();
          const uint32_t bbase = smem_u32(btiles + (use % SB) * C::kBBytes + half * (NT / 2) * 128);
          const uint32_t abuf = acol<C>(use % NA);
#pragma unroll
          for (int ks = 0; ks < 4; ++ks)
            tc::mma_ts(tmem + db * NT + half * (NT / 2), tmem + abuf + ks * 8, tc::sdesc_sw128(bbase + ks * 32),
                       idesc, (st | ks) != 0);
          tc::commit(&sdone[use % L]);
          TC_PROF_ADD(11, m3);
        }
        if (ok) tc::commit(&dfull[db]);
      }
      tc::commit(drain);  // all MMAs issued above have completed once this lands
      mbar_wait(drain, 0, a.status);
    }
  } else if (warp >= 4 && warp < 12) {
    // ------------------------------------------------------------ dequant warpgroups
    const int sub = (warp - 4) >> 2;  // 32-k half of the stage
    const int q = warp & 3;                  // tensor-memory lane quarter
    const int r = q * 32 + lane;             // weight row of this thread
    const uint32_t tlane = (uint32_t)(q * 32) << 16;
    const bool rec = (warp == 4 && lane == 0);
    (void)rec;
    int use = 0;
    bool ok = true;
    for (int item = blockIdx.x; item < total && ok; item += gridDim.x) {
      for (int st = 0; st < nstages; ++st, ++use) {
        const int s = use % SW, ab = use % NA, v = use - NA;
        TC_PROF_START(d0);
        const bool okf = mbar_wait(&wfull[s], (use / SW) & 1, a.status);
        if (rec) TC_PROF_ADD(4, d0);
        TC_PROF_START(d1);
        // A buffer use % NA is free once the MMAs of stage use - NA completed
        if (!okf || (v >= 0 && !mbar_wait(&sdone[v % L], (v / L) & 1, a.status))) {
          ok = false;
          break;
        }
        if (rec) TC_PROF_ADD(5, d1);
        TC_PROF_START(d2);
        tc::fence_after_sync();
        const uint8_t* half = wtiles + s * C::kWBytes;
        const uint8_t* meta = half + C::kHalfW;
        uint32_t zz = 0, ss;
        if constexpr (C::kAwq) {
          const uint32_t z = (meta[256 + (r >> 1)] >> (4 * (r & 1))) & 0xF;
          zz = (0x6400u | z) * 0x10001u;
          ss = (uint32_t)reinterpret_cast<const uint16_t*>(meta)[r] * 0x10001u;
        } else {
          const float sc = reinterpret_cast<const float*>(meta)[MODE == kFfn1 ? (r >> 6) : 0];
          const __half2 s2 = __float2half2_rn(sc);
          ss = *reinterpret_cast<const uint32_t*>(&s2);
        }
        uint32_t av[16];
        dequant_slice<FMT>(half, r, sub, zz, ss, av);
        tc::st_32x32b_x16(tmem + tlane + acol<C>(ab) + 16 * sub, av);
        if (rec) TC_PROF_ADD(6, d2);
        TC_PROF_START(d3);
        tc::wait_st();
        if (rec) TC_PROF_ADD(10, d3);
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&sready[use % L]);
          mbar_arrive(&wempty[s]);
        }
      }
    }
  } else if (warp >= 12) {
    // ------------------------------------------------------------ epilogue
    const int ewg = (warp - 12) >> 2;  // 16-token chunks c with c % 4 == ewg
    const int q = warp & 3;
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    float* xb = xchg + ewg * 64 * C::kXRow;
    const bool rec = (warp == 12 && lane == 0);
    (void)rec;
    int it = 0;
    for (int item = blockIdx.x; item < total; item += gridDim.x, ++it) {
      const int db = it % ND;
      int e, nt, m0, rows;
      tc_decode_item<NT>(item, tprefix, a.num_e, a.offsets, e, nt, m0, rows);
      const int row0 = a.offsets[e] + m0;
      // routing weight of token 64*i + 16*ewg + (lane & 15) of this group's chunks
      float wl[NT / 64];
#pragma unroll
      for (int i = 0; i < NT / 64; ++i) {
        const int tok = 64 * i + 16 * ewg + (lane & 15);
        wl[i] = (MODE == kFfn2 && a.row_weight && tok < rows) ? a.row_weight[row0 + tok] : 1.f;
      }
      TC_PROF_START(e0);
      if (!mbar_wait(&dfull[db], (it / ND) & 1, a.status)) break;
      if (rec) TC_PROF_ADD(7, e0);
      TC_PROF_START(e1);
      tc::fence_after_sync();
      const int nchunks = min(NT / 64, (rows - 16 * ewg + 63) / 64);  // chunks of this group with rows
      uint32_t cur[16], nxt[16];
      if (nchunks > 0) tc::ld_32x32b_x16(tmem + lane_base + db * NT + 16 * ewg, cur);
#pragma unroll 1
      for (int i = 0; i < nchunks; ++i) {
        const int c0 = 64 * i + 16 * ewg;
        tc::wait_ld();
        if (i + 1 < nchunks) tc::ld_32x32b_x16(tmem + lane_base + db * NT + c0 + 64, nxt);
        if constexpr (MODE == kFfn1) {
          // rows 0..63: gate, rows 64..127: up of the same 64 channels
          if (q >= 2) {
            float4* dst = reinterpret_cast<float4*>(xb + ((q - 2) * 32 + lane) * C::kXRow);
#pragma unroll
            for (int j = 0; j < 4; ++j)
              dst[j] = make_float4(__uint_as_float(cur[4 * j]), __uint_as_float(cur[4 * j + 1]),
                                   __uint_as_float(cur[4 * j + 2]), __uint_as_float(cur[4 * j + 3]));
          }
          named_bar(1 + ewg, 128);
          if (q < 2) {
            const float4* src = reinterpret_cast<const float4*>(xb + (q * 32 + lane) * C::kXRow);
            float u[16];
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const float4 t4 = src[j];
              u[4 * j] = t4.x;
              u[4 * j + 1] = t4.y;
              u[4 * j + 2] = t4.z;
              u[4 * j + 3] = t4.w;
            }
            const int n = nt * 64 + q * 32 + lane;
            uint16_t* orow = static_cast<uint16_t*>(a.out) + (size_t)(row0 + c0) * a.out_ld + n;
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              if (c0 + j < rows) {
                const float gv = __uint_as_float(cur[j]);
                const float hv = __fdividef(gv, 1.0f + __expf(-gv)) * u[j];
                orow[(size_t)j * a.out_ld] = __half_as_ushort(__float2half_rn(hv));
              }
            }
          }
          named_bar(1 + ewg, 128);
        } else {
          const int n = nt * kTileN + q * 32 + lane;
          float* orow = static_cast<float*>(a.out) + (size_t)(row0 + c0) * a.out_ld + n;
          float wi = wl[0];
#pragma unroll
          for (int k2 = 1; k2 < NT / 64; ++k2)
            if (k2 == i) wi = wl[k2];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const float wr = __shfl_sync(0xffffffffu, wi, j);
            if (c0 + j < rows) orow[(size_t)j * a.out_ld] = __uint_as_float(cur[j]) * wr;
          }
        }
#pragma unroll
        for (int j = 0; j < 16; ++j) cur[j] = nxt[j];
      }
      tc::fence_before_sync();
      __syncwarp();
      if (rec) TC_PROF_ADD(8, e1);
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
  static std::atomic<uint64_t> smem_set{0};  // devices with the shared-memory limit raised
  const int rc = ensure_smem_limit(kern, C::kSmem, smem_set);
  if (rc) return rc;
  return launch_k(kern, dim3(num_sms), dim3(C::kThreads), C::kSmem, st, map, a);
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

// Token tile: the smallest of 64 / 128 / 256 covering the typical expert's rows (one tile
// per expert: an MMA costs the same at any N up to 256, and at 256 the A ring is eight
// deep); 192 above (two 192-column accumulators still fit tensor memory, so the epilogue of
// one tile overlaps the MMAs of the next).  Measured on B200: 192 rows per expert run
// 5-9% faster at 256 than at 192, 384 rows faster at 192 than at 256.
// CCUT_TC_TOKEN_TILE (64, 128, 192 or 256) overrides the choice for tuning.
int tc_token_tile(int rows_per_expert) {
  static int forced = -1;
  if (forced < 0) {
    const char* e = getenv("CCUT_TC_TOKEN_TILE");
    const int v = e ? atoi(e) : 0;
    forced = (v == 64 || v == 128 || v == 192 || v == 256) ? v : 0;
  }
  if (forced) return forced;
  return rows_per_expert <= 64 ? 64 : rows_per_expert <= 128 ? 128 : rows_per_expert <= 256 ? 256 : 192;
}

int launch_tc_gemm(int fmt, int mode, int nt_tokens, const CUtensorMap& map, const TcArgs& a, int num_sms,
                   cudaStream_t st) {
  if (mode == kFfn1) {
    if (nt_tokens == 64) return launch_tc_fmt<kFfn1, 64>(fmt, map, a, num_sms, st);
    if (nt_tokens == 128) return launch_tc_fmt<kFfn1, 128>(fmt, map, a, num_sms, st);
    if (nt_tokens == 192) return launch_tc_fmt<kFfn1, 192>(fmt, map, a, num_sms, st);
    return launch_tc_fmt<kFfn1, 256>(fmt, map, a, num_sms, st);
  }
  if (nt_tokens == 64) return launch_tc_fmt<kFfn2, 64>(fmt, map, a, num_sms, st);
  if (nt_tokens == 128) return launch_tc_fmt<kFfn2, 128>(fmt, map, a, num_sms, st);
  if (nt_tokens == 192) return launch_tc_fmt<kFfn2, 192>(fmt, map, a, num_sms, st);
  return launch_tc_fmt<kFfn2, 256>(fmt, map, a, num_sms, st);
}

}  // namespace ccut
