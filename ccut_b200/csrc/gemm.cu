// gemm.cu -- dequant-fused grouped expert GEMM (gate/up + SiLU, and down).
//
// Work item = (expert, m tile of MT rows, n tile of 128 channels).  A persistent grid of
// one CTA per SM walks the items; inside a CTA
//   * warp 8 (producer) streams, per 128-k stage, the item's packed weight block(s) with
//     one bulk async copy and the MT activation row chunks (gathered through row_src) with
//     one bulk copy each, into a ring of shared-memory stages guarded by mbarriers;
//   * warps 0..7 (consumers) each own 16 output channels: they load their A fragments
//     with 128-bit shared loads, dequantize in registers (AWQ: nibble -> f16 (q - z),
//     exact, one shift + four lop3 + four f16x2 ops per eight weights; FP8: e4m3 -> f16,
//     exact), read the f16 activations with ldmatrix and issue
//     m16n8k16 tensor-core MMAs into a per-stage fp32 partial, which is then scaled by the
//     stage's group/block scale and added to the fp32 accumulator.  The weight operand is
//     therefore never rounded: (q - z) and e4m3 values are exact in f16, and the
//     scale is applied in fp32 once per 128-k group (AWQ per channel, FP8 per block).
// Epilogues: FFN1 writes silu(gate) * up as f16 rows; FFN2 writes
// row_weight[row] * acc as fp32 rows.
//
// Follows ccut/blocks/moe.py:122-141 (expert_ffn), ccut/quant/kernels.py:219-231 (SiLU),
// the dequant of ccut/quant/kernels.py:150-171 / :276-295 (restated for the g128 / block
// formats), and ccut/models/generic.py:377-378 (routing-weight scaling).
#include "kernels.cuh"

namespace ccut {

template <int FMT, int MODE, int MT>
struct GemmCfg {
  using B = Blk<FMT>;
  static constexpr int kNWarps = 8;
  static constexpr int kThreads = (kNWarps + 1) * 32;
  static constexpr int kNMat = MODE == kFfn1 ? 2 : 1;
  // AWQ down blocks are half the size of the other stages: stage two 128-k groups at once so
  // that the per-stage work (barriers, scales, partial promotion) covers as many bytes
  static constexpr int kKG = (B::kInt4 && MODE == kFfn2) ? 2 : 1;
  static constexpr int kNBlk = kNMat * kKG;  // packed blocks per stage (slots)
  static constexpr int kStageK = kTileK * kKG;
  static constexpr int kWBytes = kNBlk * B::kBytes;
  static constexpr int kXRow = kStageK * 2 + 16;  // padded row: conflict-free ldmatrix
  static constexpr int kXBytes = MT * kXRow;
  static constexpr int kStageBytes = kWBytes + kXBytes;
  // 16-row tiles (decode) run two CTAs per SM: twice the warps to hide the dequant and
  // shared-memory latencies, each with half of the shared memory.
  static constexpr int kMinBlocks = MT <= 16 ? 2 : 1;
  static constexpr int kBudget = MT <= 16 ? 100 * 1024 : 200 * 1024;
  static constexpr int kStages0 = kBudget / kStageBytes;
  static constexpr int kStages = kStages0 > 8 ? 8 : kStages0;
  // barriers, the work item of each stage slot, the item prefix over experts
  static constexpr int kHeader = 2 * 8 * kStages + 4 * kStages + 4 * (kMaxExperts + 1);
  static constexpr int kHeaderAligned = (kHeader + 127) / 128 * 128;
  static constexpr int kSmem = kHeaderAligned + kStages * kStageBytes;
  static_assert(kStages >= 2, "stage does not fit");
  static_assert(MT % 16 == 0 && MT <= 64, "MT must be 16, 32, 48 or 64");
  static_assert(kWBytes % 16 == 0 && kXRow % 16 == 0, "bulk copies need 16-byte granules");
};

template <int MT>
__device__ __forceinline__ void decode_item(int item, const int* tprefix, int num_e, const int* offsets, int ntiles,
                                            int& e, int& nt, int& m0, int& rows) {
  int lo = 0, hi = num_e - 1;  // last e with tprefix[e] <= item
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (tprefix[mid] <= item) lo = mid;
    else hi = mid - 1;
  }
  e = lo;
  const int me = offsets[e + 1] - offsets[e];
  const int mtiles = (me + MT - 1) / MT;
  const int local = item - tprefix[e];
  nt = local / mtiles;
  const int mt = local % mtiles;
  m0 = mt * MT;
  rows = min(MT, me - m0);
}

// The k loop of one item: per 128-k stage wait for the staged block(s), dequantize, issue
// the MMAs of the NB active 8-token column blocks (NB = 0: the runtime count nblk), release
// the stage and promote the scaled partial into acc.  A compile-time NB leaves no
// predicated-off MMAs in the unrolled loop.  Returns false when a bounded wait expired.
template <int FMT, int MODE, int MT, int NB>
__device__ __forceinline__ bool consume_item(const GemmArgs& a, uint8_t* stages, uint64_t* full, uint64_t* empty,
                                             int ktiles, int nblk, int warp, int lane, int ch_lo, int ch_hi,
                                             int& use,
                                             float (&acc)[GemmCfg<FMT, MODE, MT>::kNMat][MT / 8][4]) {
  using C = GemmCfg<FMT, MODE, MT>;
  using B = typename C::B;
  constexpr int S = C::kStages;
  const int nb = NB > 0 ? NB : nblk;
  constexpr int Q = C::kNBlk;  // slots: the two matrices (gate/up) or the k groups of a stage
  const int nstages = (ktiles + C::kKG - 1) / C::kKG;
  for (int kt = 0; kt < nstages; ++kt, ++use) {
    const int s = use % S;
    const int nq = C::kKG > 1 ? min(C::kKG, ktiles - kt * C::kKG) : Q;  // slots staged
    if (!mbar_wait(&full[s], (use / S) & 1, a.status)) return false;
    const uint8_t* st = stages + s * C::kStageBytes;
    const uint8_t* xs = st + C::kWBytes;
    float part[Q][MT / 8][4];
#pragma unroll
    for (int m = 0; m < Q; ++m)
#pragma unroll
      for (int b = 0; b < MT / 8; ++b)
        if (b < nb)
#pragma unroll
          for (int i = 0; i < 4; ++i) part[m][b][i] = 0.f;

    // per-stage scale (and AWQ zero-point) of this lane's two channels
    float sc_lo[Q], sc_hi[Q];
    uint32_t zp_lo[Q], zp_hi[Q];  // AWQ: f16x2 1024 + z (lo), -(64 + z) (hi)
#pragma unroll
    for (int m = 0; m < Q; ++m) {
      const uint8_t* blk = st + (m < nq ? m : 0) * B::kBytes;
      if constexpr (B::kScale == kScaleF16Row) {
        const uint16_t* sc = reinterpret_cast<const uint16_t*>(blk + B::kScaleOff);
        sc_lo[m] = __half2float(__ushort_as_half(sc[ch_lo]));
        sc_hi[m] = __half2float(__ushort_as_half(sc[ch_hi]));
      } else if constexpr (B::kScale == kScaleF32Row) {
        const float* sc = reinterpret_cast<const float*>(blk + B::kScaleOff);
        sc_lo[m] = sc[ch_lo];
        sc_hi[m] = sc[ch_hi];
      } else {
        sc_lo[m] = sc_hi[m] = reinterpret_cast<const float*>(blk + B::kScaleOff)[0];
      }
      if constexpr (B::kZeros) {
        zp_lo[m] = zero_pair_f16_1024(blk[B::kZeroOff + (ch_lo >> 1)] >> (4 * (ch_lo & 1)));
        zp_hi[m] = zero_pair_f16_neg64(blk[B::kZeroOff + (ch_hi >> 1)] >> (4 * (ch_hi & 1)));
      } else if constexpr (B::kInt4) {  // zero point 8
        zp_lo[m] = zero_pair_f16_1024(8);
        zp_hi[m] = zero_pair_f16_neg64(8);
      } else {
        zp_lo[m] = zp_hi[m] = 0;
      }
    }

#pragma unroll
    for (int kc = 0; kc < B::kChunks; ++kc) {
      uint4 raw[Q];
#pragma unroll
      for (int m = 0; m < Q; ++m)
        if (m < nq)
          raw[m] = *reinterpret_cast<const uint4*>(st + m * B::kBytes + ((warp * B::kChunks + kc) * 32 + lane) * 16);
#pragma unroll
      for (int j = 0; j < B::kStepsPerChunk; ++j) {
        uint32_t af[Q][4];
#pragma unroll
        for (int m = 0; m < Q; ++m) {
          if constexpr (B::kInt4) {
            const uint32_t wd = j == 0 ? raw[m].x : j == 1 ? raw[m].y : j == 2 ? raw[m].z : raw[m].w;
            // a0/a2: channel ch_lo (nibbles 0,4 / 2,6); a1/a3: ch_hi (nibbles 1,5 / 3,7)
            af[m][0] = nib_lo_to_f16x2_minus(wd, zp_lo[m]);
            af[m][1] = nib_hi_to_f16x2_minus(wd, zp_hi[m]);
            af[m][2] = nib_lo_to_f16x2_minus(wd >> 8, zp_lo[m]);
            af[m][3] = nib_hi_to_f16x2_minus(wd >> 8, zp_hi[m]);
          } else {
            const uint32_t w0 = j == 0 ? raw[m].x : raw[m].z;
            const uint32_t w1 = j == 0 ? raw[m].y : raw[m].w;
            af[m][0] = e4m3x2_to_f16x2(static_cast<uint16_t>(w0));
            af[m][1] = e4m3x2_to_f16x2(static_cast<uint16_t>(w0 >> 16));
            af[m][2] = e4m3x2_to_f16x2(static_cast<uint16_t>(w1));
            af[m][3] = e4m3x2_to_f16x2(static_cast<uint16_t>(w1 >> 16));
          }
        }
        const int koff = kc * B::kChunkK + j * 16;
#pragma unroll
        for (int b = 0; b < MT / 8; b += 2) {
          if (b < nb) {
            const int tok = 8 * (b + (lane >> 4)) + (lane & 7);
            const int kk = koff + ((lane >> 3) & 1) * 8;
            if constexpr (C::kKG == 1) {  // both matrices read the same activation k range
              uint32_t r0, r1, r2, r3;
              ldmatrix_x4(r0, r1, r2, r3, xs + tok * C::kXRow + kk * 2);
#pragma unroll
              for (int m = 0; m < Q; ++m) {
                mma_16816<B::kBf16>(part[m][b], af[m], r0, r1);
                if (b + 1 < nb) mma_16816<B::kBf16>(part[m][b + 1], af[m], r2, r3);
              }
            } else {  // slot m is the m-th 128-k group of the stage
#pragma unroll
              for (int m = 0; m < Q; ++m) {
                if (m < nq) {
                  uint32_t r0, r1, r2, r3;
                  ldmatrix_x4(r0, r1, r2, r3, xs + tok * C::kXRow + (kk + m * kTileK) * 2);
                  mma_16816<B::kBf16>(part[m][b], af[m], r0, r1);
                  if (b + 1 < nb) mma_16816<B::kBf16>(part[m][b + 1], af[m], r2, r3);
                }
              }
            }
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
    // promote: acc += scale * partial (fp32); k-group slots share one accumulator
#pragma unroll
    for (int m = 0; m < Q; ++m)
#pragma unroll
      for (int b = 0; b < MT / 8; ++b) {
        if (b >= nb || m >= nq) continue;
        const int ma = C::kKG > 1 ? 0 : m;
        acc[ma][b][0] = fmaf(sc_lo[m], part[m][b][0], acc[ma][b][0]);
        acc[ma][b][1] = fmaf(sc_lo[m], part[m][b][1], acc[ma][b][1]);
        acc[ma][b][2] = fmaf(sc_hi[m], part[m][b][2], acc[ma][b][2]);
        acc[ma][b][3] = fmaf(sc_hi[m], part[m][b][3], acc[ma][b][3]);
      }
  }

  return true;
}

template <int FMT, int MODE, int MT>
__global__ void __launch_bounds__(GemmCfg<FMT, MODE, MT>::kThreads, GemmCfg<FMT, MODE, MT>::kMinBlocks)
    moe_gemm_kernel(GemmArgs a) {
  pdl_wait();
  pdl_trigger();
  using C = GemmCfg<FMT, MODE, MT>;
  using B = typename C::B;
  constexpr int S = C::kStages;
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem);
  uint64_t* empty = full + S;
  volatile int* slot_item = reinterpret_cast<int*>(smem + 16 * S);  // item whose first stage the slot holds
  int* tprefix = reinterpret_cast<int*>(smem + 20 * S);
  uint8_t* stages = smem + C::kHeaderAligned;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ntiles = a.N / kTileN, ktiles = a.K / kTileK;

  if (warp == 0) {  // item prefix over experts: tiles(e) = ceil(M_e / MT) * ntiles
    int carry = 0;
    for (int b = 0; b < a.num_e; b += 32) {
      const int e = b + lane;
      const int me = e < a.num_e ? a.offsets[e + 1] - a.offsets[e] : 0;
      const int c = ((me + MT - 1) / MT) * ntiles;
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
  if (threadIdx.x == 32) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], C::kNWarps);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  const int total = tprefix[a.num_e];

  if (warp == C::kNWarps) {
    // ---------------- producer ----------------
    // Work items go out in increasing order: CTA c takes item c, then either fetches the
    // next one from the counter a.sched[0] (dynamic: CTAs that finish early take more, so
    // the SMs end at about the same time whatever their speed or item count) or takes
    // c + grid, c + 2 grid, ... (static).
    // The item id travels to the consumers in the slot of the item's first stage, published
    // by that stage's full-barrier arrival; -1 ends the walk.
    int use = 0;
    bool ok = true;
    // The first wave is static (CTA c starts with item c, so a small launch spreads over
    // distinct SMs rather than pairing up on the first CTAs to fetch).
    int item = (int)blockIdx.x;
    while (ok && item < total) {
      int next = 0;  // lane 0: the next item, fetched now and read after this item's stages
      if (a.sched != nullptr && lane == 0) next = (int)gridDim.x + atomicAdd(&a.sched[0], 1);
      int e, nt, m0, rows;
      decode_item<MT>(item, tprefix, a.num_e, a.offsets, ntiles, e, nt, m0, rows);
      const int row0 = a.offsets[e] + m0;
      int src[MT / 32 + 1];
#pragma unroll
      for (int i = 0; i * 32 < MT; ++i) {
        const int r = lane + 32 * i;
        src[i] = r < rows ? (a.row_src ? a.row_src[row0 + r] : row0 + r) : 0;
      }
      const uint8_t* wb = a.w + (size_t)e * a.expert_stride + (size_t)nt * ktiles * C::kNMat * B::kBytes;
      const int nstages = (ktiles + C::kKG - 1) / C::kKG;
      for (int kt = 0; kt < nstages; ++kt, ++use) {
        const int nq = C::kKG > 1 ? min(C::kKG, ktiles - kt * C::kKG) : 1;  // k groups staged
        const uint32_t wbytes = nq * C::kNMat * B::kBytes, xbytes = nq * kTileK * 2;
        const int s = use % S;
        const uint32_t ph = (use / S) & 1;
        if (!mbar_wait(&empty[s], ph ^ 1, a.status)) {
          ok = false;
          break;
        }
        uint8_t* st = stages + s * C::kStageBytes;
        if (lane == 0) {
          if (kt == 0) slot_item[s] = item;
          mbar_arrive_expect_tx(&full[s], wbytes + rows * xbytes);
          bulk_g2s(st, wb + (size_t)kt * C::kWBytes, wbytes, &full[s]);
        }
        __syncwarp();
#pragma unroll
        for (int i = 0; i * 32 < MT; ++i) {
          const int r = lane + 32 * i;
          if (r < rows)
            bulk_g2s(st + C::kWBytes + r * C::kXRow, a.x + (size_t)src[i] * a.x_ld + kt * C::kStageK, xbytes,
                     &full[s]);
        }
      }
      item = a.sched != nullptr ? __shfl_sync(0xffffffffu, next, 0) : item + (int)gridDim.x;
    }
    if (ok) {  // end marker: the next slot carries item -1 and no bytes
      const int s = use % S;
      if (mbar_wait(&empty[s], ((use / S) & 1) ^ 1, a.status)) {
        if (lane == 0) {
          slot_item[s] = -1;
          mbar_arrive(&full[s]);
        }
      } else {
        ok = false;
      }
    }
    if (!ok && lane == 0) {  // let the copies already issued land before the CTA exits
      for (int u = use > S ? use - S : 0; u < use; ++u) mbar_wait(&full[u % S], (u / S) & 1, nullptr);
    }
    // The last CTA to finish fetching leaves the counters zero for the next launch.
    if (a.sched != nullptr && lane == 0 && atomicAdd(&a.sched[1], 1) == (int)gridDim.x - 1) {
      a.sched[0] = 0;
      a.sched[1] = 0;
    }
    return;
  }

  // ---------------- consumers ----------------
  const int g = lane >> 2, t = lane & 3;
  const int ch_lo = warp * 16 + g, ch_hi = ch_lo + 8;  // channels within the 128-tile
  int use = 0;
  while (true) {
    {  // the item of the next stage (its full barrier completes before the slot is read)
      const int s = use % S;
      if (!mbar_wait(&full[s], (use / S) & 1, a.status)) return;
    }
    const int item = slot_item[use % S];
    if (item < 0) break;
    int e, nt, m0, rows;
    decode_item<MT>(item, tprefix, a.num_e, a.offsets, ntiles, e, nt, m0, rows);
    const int nblk = (rows + 7) >> 3;  // 8-token MMA column blocks in use
    float acc[C::kNMat][MT / 8][4];
#pragma unroll
    for (int m = 0; m < C::kNMat; ++m)
#pragma unroll
      for (int b = 0; b < MT / 8; ++b)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[m][b][i] = 0.f;

    bool alive;
    if constexpr (MT == 16) {  // one or two active column blocks
      alive = nblk == 1
                  ? consume_item<FMT, MODE, MT, 1>(a, stages, full, empty, ktiles, nblk, warp, lane, ch_lo, ch_hi, use, acc)
                  : consume_item<FMT, MODE, MT, 2>(a, stages, full, empty, ktiles, nblk, warp, lane, ch_lo, ch_hi, use, acc);
    } else if constexpr (MT == 32) {
      alive = nblk == 1
                  ? consume_item<FMT, MODE, MT, 1>(a, stages, full, empty, ktiles, nblk, warp, lane, ch_lo, ch_hi, use, acc)
                  : consume_item<FMT, MODE, MT, 0>(a, stages, full, empty, ktiles, nblk, warp, lane, ch_lo, ch_hi, use, acc);
    } else {
      alive = consume_item<FMT, MODE, MT, 0>(a, stages, full, empty, ktiles, nblk, warp, lane, ch_lo, ch_hi, use, acc);
    }
    if (!alive) return;

    // ---------------- epilogue ----------------
    const int row0 = a.offsets[e] + m0;
    const int n_lo = nt * kTileN + ch_lo, n_hi = n_lo + 8;
#pragma unroll
    for (int b = 0; b < MT / 8; ++b) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int tok = 8 * b + 2 * t + (i & 1);
        if (tok < rows) {
          const int n = i < 2 ? n_lo : n_hi;
          const size_t o = (size_t)(row0 + tok) * a.out_ld + n;
          if constexpr (MODE == kFfn1) {
            const float h = silu(acc[0][b][i]) * acc[1][b][i];
            uint16_t hv;
            if constexpr (B::kBf16) hv = __bfloat16_as_ushort(__float2bfloat16_rn(h));
            else hv = __half_as_ushort(__float2half_rn(h));
            static_cast<uint16_t*>(a.out)[o] = hv;
          } else {
            const float wr = a.row_weight ? a.row_weight[row0 + tok] : 1.f;
            if (a.out_bf16)
              static_cast<uint16_t*>(a.out)[o] = __bfloat16_as_ushort(__float2bfloat16_rn(acc[0][b][i] * wr));
            else
              static_cast<float*>(a.out)[o] = acc[0][b][i] * wr;
          }
        }
      }
    }
  }
}


template <int FMT, int MODE, int MT>
static int launch_gemm_t(const GemmArgs& a, int num_sms, cudaStream_t st) {
  using C = GemmCfg<FMT, MODE, MT>;
  auto kern = moe_gemm_kernel<FMT, MODE, MT>;
  static std::atomic<uint64_t> smem_set{0};  // devices with the shared-memory limit raised
  const int rc = ensure_smem_limit(kern, C::kSmem, smem_set);
  if (rc) return rc;
  return launch_k(kern, dim3(num_sms * C::kMinBlocks), dim3(C::kThreads), C::kSmem, st, a);
}

template <int FMT, int MODE>
static int launch_gemm_mt(int mt, const GemmArgs& a, int num_sms, cudaStream_t st) {
  if (mt <= 16) return launch_gemm_t<FMT, MODE, 16>(a, num_sms, st);
  if (mt <= 32) return launch_gemm_t<FMT, MODE, 32>(a, num_sms, st);
  return launch_gemm_t<FMT, MODE, 64>(a, num_sms, st);
}

// Token-tile height: 16 (two CTAs per SM) and 32 cover decode batches in one tile; 64
// halves weight re-reads for larger batches.
int launch_gemm(int fmt, int mode, int mt, const GemmArgs& a, int num_sms, cudaStream_t st) {
  switch (fmt) {
    case CCUT_FMT_AWQ_INT4_G128:
      return mode == kFfn1 ? launch_gemm_mt<CCUT_FMT_AWQ_INT4_G128, kFfn1>(mt, a, num_sms, st)
                           : launch_gemm_mt<CCUT_FMT_AWQ_INT4_G128, kFfn2>(mt, a, num_sms, st);
    case CCUT_FMT_INT4_SYM_G128:
      return mode == kFfn1 ? launch_gemm_mt<CCUT_FMT_INT4_SYM_G128, kFfn1>(mt, a, num_sms, st)
                           : launch_gemm_mt<CCUT_FMT_INT4_SYM_G128, kFfn2>(mt, a, num_sms, st);
    case CCUT_FMT_FP8_E4M3_CH:
      return mode == kFfn1 ? launch_gemm_mt<CCUT_FMT_FP8_E4M3_CH, kFfn1>(mt, a, num_sms, st)
                           : launch_gemm_mt<CCUT_FMT_FP8_E4M3_CH, kFfn2>(mt, a, num_sms, st);
    default:
      return mode == kFfn1 ? launch_gemm_mt<CCUT_FMT_FP8_E4M3_B128, kFfn1>(mt, a, num_sms, st)
                           : launch_gemm_mt<CCUT_FMT_FP8_E4M3_B128, kFfn2>(mt, a, num_sms, st);
  }
}

}  // namespace ccut
