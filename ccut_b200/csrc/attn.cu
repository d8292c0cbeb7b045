// attn.cu -- GQA attention (flash-decoding, split over the kv range) and RMSNorm.
//
// GQA: q bf16 [B, Hq, S, D], k / v bf16 [B, Hkv, L, D] -> o [B, Hq, S, D] (fp32 or bf16),
// query head h reading kv head h / (Hq / Hkv).  Scores are fp32 q . k * scale, optionally
// soft-capped (tanh(s / c) * c), causally masked (query i sees kv positions
// <= causal_start + i) and softmax-normalised; the output is probs @ v.  This is
// ccut/blocks/attn_gqa.py:127-153 (gqa_attention_fast, the function the reference's
// attention layer calls at ccut/models/generic.py:343) with the mask of build_causal_mask
// (:65-73) and the softcap of gqa_attention (:76-124).
//
// Work: a CTA takes 16 query rows of one (batch, kv head) -- the query heads that share
// the kv head, row r = (s, g) with s = r / G, g = r % G -- and one split of the kv range;
// the 16 rows are the M of m16n8k16 bf16 tensor-core MMAs (S = Q K^T, then O += P V with P
// split into bf16 hi + lo parts), see gqa_attn_kernel.  With one split the CTA writes
// o = acc / max(l, 1e-30); with several it writes (m, l, acc) and gqa_combine_kernel merges
// the splits.  Bound: HBM (K and V read once per (batch, kv head, split); the query rows of
// a kv head share them).
//
// RMSNorm: y = x * (mean(x^2) + eps)^-1/2 * w per row in fp32 (ccut/blocks/norm.py:14-26).
// RoPE: half-rotation rotary embedding (ccut/blocks/rope.py:130-175).
#include <math.h>

#include "host.cuh"

namespace ccut {

constexpr int kAttnTile = 64;  // kv positions per staged tile

__device__ __forceinline__ float bf16_to_f32(uint16_t b) { return __uint_as_float((uint32_t)b << 16); }

// ---- tensor-core tiles ------------------------------------------------------------------
__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3,
                                                  const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(smem_u32(p)));
}
// (bf16(a), bf16(b)) and the bf16 residuals (a - bf16(a), b - bf16(b)), packed low = a
__device__ __forceinline__ void split_bf16x2(float a, float b, uint32_t& hi, uint32_t& lo) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  const __nv_bfloat162 r = __floats2bfloat162_rn(a - __low2float(h), b - __high2float(h));
  hi = *reinterpret_cast<const uint32_t*>(&h);
  lo = *reinterpret_cast<const uint32_t*>(&r);
}

constexpr int kTcRows = 16;  // query rows per CTA (the MMA's M)
constexpr int kTcWarps = 4;  // warps per CTA, each streaming its own kv tiles
constexpr int kTcTile = 16;  // kv positions per warp tile

template <int D>
struct TcAttnSmem {
  static constexpr int kRow = D + 8;  // padded row (elements): conflict-free ldmatrix
  static constexpr int kTileElems = kTcTile * kRow;
  static constexpr int kStages = 3;                     // K/V tiles per warp: one in use, two in flight
  static constexpr int kWarpElems = kStages * 2 * kTileElems;
  static constexpr int kQElems = kTcRows * kRow;
  static constexpr size_t kLoopBytes = (size_t)(kQElems + kTcWarps * kWarpElems) * 2;
  static constexpr size_t kMergeBytes = (size_t)kTcWarps * kTcRows * (D + 2) * 4;  // aliases the tiles
  static constexpr size_t kBytes = kLoopBytes > kMergeBytes ? kLoopBytes : kMergeBytes;
  static_assert((kRow * 2) % 16 == 0 && (kQElems * 2) % 16 == 0 && (kTileElems * 2) % 16 == 0, "16-byte rows");
};

// Tensor-core tiles on the m16n8k16 bf16 MMA (fp32 accumulate): the CTA's 16 query rows are
// the A operand of S = Q K^T (K rows read with ldmatrix as B fragments); the probabilities
// P, split into bf16 hi + lo parts so that P V keeps ~16 bits, are the A operand of O += P V
// (V read with ldmatrix.trans).  Each warp streams its own tiles of 16 kv positions
// (tile j of the CTA's range goes to warp j % 4) through a three-deep cp.async ring and keeps
// its own online softmax (running max and sum of rows g and g + 8, fp32 O fragments); the
// four warp states are merged through shared memory at the end.
//
// The body serves two kernels.  gqa_attn_kernel: batch row b reads k / v at b's slice of
// [B, Hkv, L, D] with one causal offset for all rows.  gqa_attn_pool_kernel (POOL): batch row
// b reads slot slots[b] of a cache pool (slots slot_stride elements apart, kv head h at
// h * L * D inside a slot) with causal offset starts[b], so one launch serves sequences of
// different lengths; a slot outside [0, num_slots) or a negative offset reads nothing and its
// rows come out zero.
template <int D, bool OUT_BF16, bool POOL>
__device__ __forceinline__ void gqa_attn_body(
    const uint16_t* __restrict__ q, const uint16_t* __restrict__ k, const uint16_t* __restrict__ v, int Hq, int Hkv,
    int S, int L, int causal_start, float scale, float softcap, int splits, int tiles_per_split,
    void* __restrict__ out, float* __restrict__ part, const int* __restrict__ slots, const int* __restrict__ starts,
    long long slot_stride, int num_slots) {
  pdl_wait();
  pdl_trigger();
  using SM = TcAttnSmem<D>;
  constexpr int KS = D / 16;  // k steps of Q K^T; dim-tile pairs of P V
  extern __shared__ __align__(128) uint8_t attn_smem[];
  uint16_t* qs = reinterpret_cast<uint16_t*>(attn_smem);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int G = Hq / Hkv, nrows = G * S;
  const int bh = blockIdx.y, b = bh / Hkv, kvh = bh % Hkv;
  const int r0 = blockIdx.x * kTcRows;
  const int split = blockIdx.z;
  const int k0 = split * tiles_per_split * kAttnTile;
  int k1 = min(L, k0 + tiles_per_split * kAttnTile);
  size_t kv_off = (size_t)bh * L * D;
  if constexpr (POOL) {
    const int slot = slots[b];
    causal_start = starts[b];
    const bool valid = slot >= 0 && slot < num_slots && causal_start >= 0;
    if (!valid) {
      k1 = 0;  // nothing to read: the rows come out zero
      causal_start = 0;
    }
    kv_off = (valid ? (size_t)slot * (size_t)slot_stride : (size_t)0) + (size_t)kvh * L * D;
  }
  if (causal_start >= 0) {  // the CTA's last row sees up to causal_start + s_last
    const int r_last = min(nrows, r0 + kTcRows) - 1;
    k1 = min(k1, causal_start + r_last / G + 1);
  }
  // Q rows -> shared memory (zero rows past the end), then A fragments in registers
  for (int c = threadIdx.x; c < kTcRows * (D / 8); c += blockDim.x) {
    const int rr = c / (D / 8), dc = (c % (D / 8)) * 8, r = r0 + rr;
    uint4 val = make_uint4(0, 0, 0, 0);
    if (r < nrows) {
      const int s = r / G, h = kvh * G + r % G;
      val = *reinterpret_cast<const uint4*>(q + (((size_t)b * Hq + h) * S + s) * D + dc);
    }
    *reinterpret_cast<uint4*>(qs + rr * SM::kRow + dc) = val;
  }
  __syncthreads();
  uint32_t qa[KS][4];
#pragma unroll
  for (int ks = 0; ks < KS; ++ks)
    ldmatrix_x4(qa[ks][0], qa[ks][1], qa[ks][2], qa[ks][3],
                qs + ((lane & 7) + ((lane >> 3) & 1) * 8) * SM::kRow + ks * 16 + (lane >> 4) * 8);
  int lim[2];  // last visible kv position of rows g and g + 8
#pragma unroll
  for (int i = 0; i < 2; ++i) lim[i] = causal_start >= 0 ? causal_start + (r0 + g + 8 * i) / G : L - 1;

  float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
  float o[2 * KS][4];
#pragma unroll
  for (int dn = 0; dn < 2 * KS; ++dn)
#pragma unroll
    for (int i = 0; i < 4; ++i) o[dn][i] = 0.f;
  uint16_t* wb = qs + SM::kQElems + warp * SM::kWarpElems;  // [stage][K, V][16][kRow]
  const uint16_t* kg = k + kv_off;
  const uint16_t* vg = v + kv_off;
  const int ntiles = k1 > k0 ? (k1 - k0 + kTcTile - 1) / kTcTile : 0;
  auto issue = [&](int tile, int buf) {
    const int p0 = k0 + tile * kTcTile;
    uint16_t* kd = wb + buf * 2 * SM::kTileElems;
    uint16_t* vd = kd + SM::kTileElems;
    for (int c = lane; c < kTcTile * (D / 8); c += 32) {
      const int pr = c / (D / 8), dc = (c % (D / 8)) * 8, pos = p0 + pr;
      const bool ok = pos < k1;
      const size_t off = (size_t)(ok ? pos : 0) * D + dc;
      cp_async16(kd + pr * SM::kRow + dc, kg + off, ok);
      cp_async16(vd + pr * SM::kRow + dc, vg + off, ok);
    }
  };
  // one commit group per tile slot (empty past the end), so that wait_group<kStages - 1>
  // always means "this iteration's tile has landed"
#pragma unroll
  for (int st = 0; st < SM::kStages - 1; ++st) {
    if (warp + st * kTcWarps < ntiles) issue(warp + st * kTcWarps, st);
    cp_async_commit();
  }
  int buf = 0;
  for (int jt = warp; jt < ntiles; jt += kTcWarps) {
    const int jn = jt + (SM::kStages - 1) * kTcWarps;
    if (jn < ntiles) issue(jn, (buf + SM::kStages - 1) % SM::kStages);
    cp_async_commit();
    cp_async_wait<SM::kStages - 1>();
    __syncwarp();
    const uint16_t* kd = wb + buf * 2 * SM::kTileElems;
    const uint16_t* vd = kd + SM::kTileElems;
    // S = Q K^T over 16 positions (two n8 tiles)
    float sc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
      const int mi = lane >> 3;
      uint32_t b0, b1, b2, b3;
      ldmatrix_x4(b0, b1, b2, b3, kd + ((mi >> 1) * 8 + (lane & 7)) * SM::kRow + ks * 16 + (mi & 1) * 8);
      mma_16816<true>(sc[0], qa[ks], b0, b1);
      mma_16816<true>(sc[1], qa[ks], b2, b3);
    }
    // scale, cap, mask; element (n, i): row g + 8 (i >> 1), position p0 + 8 n + 2 t + (i & 1)
    const int p0 = k0 + jt * kTcTile;
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int n = 0; n < 2; ++n)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float x = sc[n][i] * scale;
        if (softcap > 0.f) x = tanhf(x / softcap) * softcap;
        const int pos = p0 + 8 * n + 2 * t + (i & 1);
        if (pos >= k1 || pos > lim[i >> 1]) x = -INFINITY;
        sc[n][i] = x;
        mx[i >> 1] = fmaxf(mx[i >> 1], x);
      }
    float mnew[2], alpha[2], rs[2] = {0.f, 0.f};
#pragma unroll
    for (int ri = 0; ri < 2; ++ri) {
      mx[ri] = fmaxf(mx[ri], __shfl_xor_sync(0xffffffffu, mx[ri], 1));
      mx[ri] = fmaxf(mx[ri], __shfl_xor_sync(0xffffffffu, mx[ri], 2));
      mnew[ri] = fmaxf(m[ri], mx[ri]);
      alpha[ri] = mnew[ri] == -INFINITY ? 1.f : expf(m[ri] - mnew[ri]);  // 0 after an all-masked start
    }
#pragma unroll
    for (int n = 0; n < 2; ++n)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int ri = i >> 1;
        const float p = mnew[ri] == -INFINITY ? 0.f : expf(sc[n][i] - mnew[ri]);
        sc[n][i] = p;
        rs[ri] += p;
      }
#pragma unroll
    for (int ri = 0; ri < 2; ++ri) {
      rs[ri] += __shfl_xor_sync(0xffffffffu, rs[ri], 1);
      rs[ri] += __shfl_xor_sync(0xffffffffu, rs[ri], 2);
      l[ri] = l[ri] * alpha[ri] + rs[ri];
      m[ri] = mnew[ri];
    }
#pragma unroll
    for (int dn = 0; dn < 2 * KS; ++dn) {
      o[dn][0] *= alpha[0];
      o[dn][1] *= alpha[0];
      o[dn][2] *= alpha[1];
      o[dn][3] *= alpha[1];
    }
    // P as the A operand (the two n8 score tiles form one k16 step), hi and lo parts
    uint32_t ph[4], pl[4];
    split_bf16x2(sc[0][0], sc[0][1], ph[0], pl[0]);
    split_bf16x2(sc[0][2], sc[0][3], ph[1], pl[1]);
    split_bf16x2(sc[1][0], sc[1][1], ph[2], pl[2]);
    split_bf16x2(sc[1][2], sc[1][3], ph[3], pl[3]);
#pragma unroll
    for (int dp = 0; dp < KS; ++dp) {
      const int mi = lane >> 3;
      uint32_t b0, b1, b2, b3;
      ldmatrix_x4_trans(b0, b1, b2, b3, vd + ((mi & 1) * 8 + (lane & 7)) * SM::kRow + dp * 16 + (mi >> 1) * 8);
      mma_16816<true>(o[2 * dp], ph, b0, b1);
      mma_16816<true>(o[2 * dp], pl, b0, b1);
      mma_16816<true>(o[2 * dp + 1], ph, b2, b3);
      mma_16816<true>(o[2 * dp + 1], pl, b2, b3);
    }
    __syncwarp();  // this stage is refilled by the next iteration's issue
    buf = (buf + 1) % SM::kStages;
  }
  // merge the four warp states (the merge area aliases the tile buffers)
  __syncthreads();
  float* mg = reinterpret_cast<float*>(attn_smem);
  {
    float* wm = mg + (size_t)warp * kTcRows * (D + 2);
#pragma unroll
    for (int dn = 0; dn < 2 * KS; ++dn) {
      wm[g * (D + 2) + 2 + dn * 8 + 2 * t] = o[dn][0];
      wm[g * (D + 2) + 3 + dn * 8 + 2 * t] = o[dn][1];
      wm[(g + 8) * (D + 2) + 2 + dn * 8 + 2 * t] = o[dn][2];
      wm[(g + 8) * (D + 2) + 3 + dn * 8 + 2 * t] = o[dn][3];
    }
    if (t == 0) {
      wm[g * (D + 2)] = m[0];
      wm[g * (D + 2) + 1] = l[0];
      wm[(g + 8) * (D + 2)] = m[1];
      wm[(g + 8) * (D + 2) + 1] = l[1];
    }
  }
  __syncthreads();
  const size_t rows_total = (size_t)(gridDim.y / Hkv) * Hq * S;  // B * Hq * S
  for (int idx = threadIdx.x; idx < kTcRows * D; idx += blockDim.x) {
    const int rr = idx / D, dd = idx % D, r = r0 + rr;
    if (r >= nrows) continue;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kTcWarps; ++w) M = fmaxf(M, mg[(w * kTcRows + rr) * (D + 2)]);
    float Ls = 0.f, ov = 0.f;
    if (M > -INFINITY) {
#pragma unroll
      for (int w = 0; w < kTcWarps; ++w) {
        const float* row = mg + (w * kTcRows + rr) * (D + 2);
        const float e = expf(row[0] - M);  // 0 for a warp that saw nothing
        Ls = fmaf(row[1], e, Ls);
        ov = fmaf(row[2 + dd], e, ov);
      }
    }
    const int s = r / G, h = kvh * G + r % G;
    const size_t orow = ((size_t)b * Hq + h) * S + s;
    if (splits == 1) {
      const float val = ov / fmaxf(Ls, 1e-30f);
      if constexpr (OUT_BF16) static_cast<__nv_bfloat16*>(out)[orow * D + dd] = __float2bfloat16_rn(val);
      else static_cast<float*>(out)[orow * D + dd] = val;
    } else {
      float* p = part + ((size_t)split * rows_total + orow) * (D + 2);
      if (dd == 0) {
        p[0] = M;
        p[1] = Ls;
      }
      p[2 + dd] = ov;
    }
  }
}

template <int D, bool OUT_BF16>
__global__ void __launch_bounds__(kTcWarps * 32) gqa_attn_kernel(
    const uint16_t* __restrict__ q, const uint16_t* __restrict__ k, const uint16_t* __restrict__ v, int Hq, int Hkv,
    int S, int L, int causal_start, float scale, float softcap, int splits, int tiles_per_split,
    void* __restrict__ out, float* __restrict__ part) {
  gqa_attn_body<D, OUT_BF16, false>(q, k, v, Hq, Hkv, S, L, causal_start, scale, softcap, splits, tiles_per_split,
                                    out, part, nullptr, nullptr, 0, 0);
}

template <int D, bool OUT_BF16>
__global__ void __launch_bounds__(kTcWarps * 32) gqa_attn_pool_kernel(
    const uint16_t* __restrict__ q, const uint16_t* __restrict__ k, const uint16_t* __restrict__ v, int Hq, int Hkv,
    int S, int L, float scale, float softcap, int splits, int tiles_per_split, void* __restrict__ out,
    float* __restrict__ part, const int* __restrict__ slots, const int* __restrict__ starts, long long slot_stride,
    int num_slots) {
  gqa_attn_body<D, OUT_BF16, true>(q, k, v, Hq, Hkv, S, L, 0, scale, softcap, splits, tiles_per_split, out, part,
                                   slots, starts, slot_stride, num_slots);
}

// Merge of the kv splits: one warp per output row.
template <int D, bool OUT_BF16>
__global__ void __launch_bounds__(256) gqa_combine_kernel(const float* __restrict__ part, int rows, int splits,
                                                          void* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  constexpr int DL = D / 32;
  const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (row >= rows) return;
  float M = -INFINITY;
  for (int sp = 0; sp < splits; ++sp) M = fmaxf(M, part[((size_t)sp * rows + row) * (D + 2)]);
  float Lsum = 0.f, o[DL];
#pragma unroll
  for (int j = 0; j < DL; ++j) o[j] = 0.f;
  if (M > -INFINITY) {
    for (int sp = 0; sp < splits; ++sp) {
      const float* p = part + ((size_t)sp * rows + row) * (D + 2);
      const float w = expf(p[0] - M);  // 0 for a split that saw nothing (m = -inf)
      Lsum = fmaf(p[1], w, Lsum);
#pragma unroll
      for (int j = 0; j < DL; ++j) o[j] = fmaf(p[2 + lane * DL + j], w, o[j]);
    }
  }
  const float inv = 1.f / fmaxf(Lsum, 1e-30f);
#pragma unroll
  for (int j = 0; j < DL; ++j) {
    const size_t idx = (size_t)row * D + lane * DL + j;
    if constexpr (OUT_BF16) static_cast<__nv_bfloat16*>(out)[idx] = __float2bfloat16_rn(o[j] * inv);
    else static_cast<float*>(out)[idx] = o[j] * inv;
  }
}

// ---- MLA in the latent space (DeepSeek-V2 / V3, the absorbed form) -----------------------
// q [B, S*H, 576] fp32, row r = s * H + h: q_nope of head h folded through k_up (512 latent
// features), then the rotated q_pe (64).  kv [B, L, 576] bf16, one row per position: the
// latent c (512), then the rotated k_pe (64).  out o_lat [B, S*H, 512] =
// softmax(q . kv^T * scale, causal) @ kv[:, :512].  This is ccut/blocks/attn_mla.py:85-167
// (mla_decode / mla_prefill) with the up-projections outside the kernel: the scores
// (c k_up_h) . q_nope + k_pe . q_pe equal (q_nope k_up_h^T) . c + q_pe . k_pe, and the output
// probs @ (c v_up_h) equals (probs @ c) v_up_h.
//
// Work: a CTA takes 16 query rows and one split of the kv range of one sequence; every row
// of the CTA reads the same latent rows, so each position's 1152 bytes are read once per
// (sequence, split).  Per 16-position tile, staged through a three-deep cp.async ring
// shared by the CTA, the four warps split both products along the features: warp w computes
// S over key features [144 w, 144 w + 144) (q split into bf16 hi + lo parts, so that q keeps
// ~16 bits), the four partial S tiles are summed in warp order through shared memory (every
// warp then holds the same S and runs the same online softmax), and warp w accumulates
// O += P V for value features [128 w, 128 w + 128) (P split into hi + lo as in the GQA
// kernel).  Splits are merged by gqa_combine_kernel<512>.  mla_attn_pool_kernel (POOL): batch
// row b reads slot slots[b] of a latent-cache pool (slots slot_stride elements apart, L rows
// of 576 in each) with causal offset starts[b], so one launch serves sequences of different
// lengths; a slot outside [0, num_slots) or a negative offset reads nothing and its rows come
// out zero.
constexpr int kMlaR = 512, kMlaP = 64, kMlaK = kMlaR + kMlaP;  // latent rank, rope features, key width
constexpr int kMlaWarps = 4;
constexpr int kMlaKS = kMlaK / kMlaWarps / 16;  // k16 steps of S per warp (9)
constexpr int kMlaVW = kMlaR / kMlaWarps;       // value features per warp (128)
constexpr int kMlaTile = 16;                    // kv positions per staged tile
constexpr int kMlaStages = 3;
constexpr int kMlaRow = kMlaK + 8;  // padded shared-memory row (elements): conflict-free ldmatrix

struct MlaSmem {
  static constexpr int kQElems = kTcRows * kMlaRow;     // one of the q hi / lo planes
  static constexpr int kTileElems = kMlaTile * kMlaRow;  // one ring stage
  static constexpr size_t kRedBytes = (size_t)kMlaWarps * 32 * 8 * sizeof(float);  // partial S fragments
  static constexpr size_t kBytes = (size_t)(2 * kQElems + kMlaStages * kTileElems) * 2 + kRedBytes;
  static_assert((kMlaRow * 2) % 16 == 0 && (kQElems * 2) % 16 == 0 && (kTileElems * 2) % 16 == 0, "16-byte rows");
  static_assert(kMlaKS * 16 * kMlaWarps == kMlaK && kMlaVW % 16 == 0, "feature split");
};

template <bool OUT_BF16, bool POOL>
__device__ __forceinline__ void mla_attn_body(
    const float* __restrict__ q, const uint16_t* __restrict__ kv, int H, int S, int L, int causal_start, float scale,
    int splits, int tiles_per_split, void* __restrict__ out, float* __restrict__ part, const int* __restrict__ slots,
    const int* __restrict__ starts, long long slot_stride, int num_slots) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ __align__(128) uint8_t mla_smem[];
  uint16_t* qhi = reinterpret_cast<uint16_t*>(mla_smem);
  uint16_t* qlo = qhi + MlaSmem::kQElems;
  uint16_t* ring = qlo + MlaSmem::kQElems;
  float* red = reinterpret_cast<float*>(ring + kMlaStages * MlaSmem::kTileElems);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int nrows = S * H;
  const int b = blockIdx.y, r0 = blockIdx.x * kTcRows, split = blockIdx.z;
  const int k0 = split * tiles_per_split * kMlaTile;
  int k1 = min(L, k0 + tiles_per_split * kMlaTile);
  size_t kv_off = (size_t)b * L * kMlaK;
  if constexpr (POOL) {
    const int slot = slots[b];
    causal_start = starts[b];
    const bool valid = slot >= 0 && slot < num_slots && causal_start >= 0;
    if (!valid) {
      k1 = 0;  // nothing to read: the rows come out zero
      causal_start = 0;
    }
    kv_off = valid ? (size_t)slot * (size_t)slot_stride : (size_t)0;
  }
  if (causal_start >= 0) {  // the CTA's last row sees up to causal_start + s_last
    const int r_last = min(nrows, r0 + kTcRows) - 1;
    k1 = min(k1, causal_start + r_last / H + 1);
  }
  const int ntiles = k1 > k0 ? (k1 - k0 + kMlaTile - 1) / kMlaTile : 0;
  const uint16_t* kvg = kv + kv_off;
  auto issue = [&](int tile) {  // tile -> ring stage tile % kMlaStages, zero-filled past k1
    const int p0 = k0 + tile * kMlaTile;
    uint16_t* dst = ring + (tile % kMlaStages) * MlaSmem::kTileElems;
    for (int c = threadIdx.x; c < kMlaTile * (kMlaK / 8); c += blockDim.x) {
      const int pr = c / (kMlaK / 8), dc = (c % (kMlaK / 8)) * 8, pos = p0 + pr;
      const bool ok = pos < k1;
      cp_async16(dst + pr * kMlaRow + dc, kvg + (size_t)(ok ? pos : 0) * kMlaK + dc, ok);
    }
  };
#pragma unroll
  for (int st = 0; st < kMlaStages - 1; ++st) {
    if (st < ntiles) issue(st);
    cp_async_commit();
  }
  // the CTA's 16 query rows -> bf16 hi / lo planes in shared memory (zero rows past the end)
  for (int c = threadIdx.x; c < kTcRows * (kMlaK / 4); c += blockDim.x) {
    const int rr = c / (kMlaK / 4), dc = (c % (kMlaK / 4)) * 4, r = r0 + rr;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (r < nrows) v = *reinterpret_cast<const float4*>(q + ((size_t)b * nrows + r) * kMlaK + dc);
    uint32_t h0, l0, h1, l1;
    split_bf16x2(v.x, v.y, h0, l0);
    split_bf16x2(v.z, v.w, h1, l1);
    *reinterpret_cast<uint2*>(qhi + rr * kMlaRow + dc) = make_uint2(h0, h1);
    *reinterpret_cast<uint2*>(qlo + rr * kMlaRow + dc) = make_uint2(l0, l1);
  }
  __syncthreads();
  uint32_t qah[kMlaKS][4], qal[kMlaKS][4];
#pragma unroll
  for (int kk = 0; kk < kMlaKS; ++kk) {
    const int off = ((lane & 7) + ((lane >> 3) & 1) * 8) * kMlaRow + (warp * kMlaKS + kk) * 16 + (lane >> 4) * 8;
    ldmatrix_x4(qah[kk][0], qah[kk][1], qah[kk][2], qah[kk][3], qhi + off);
    ldmatrix_x4(qal[kk][0], qal[kk][1], qal[kk][2], qal[kk][3], qlo + off);
  }
  int lim[2];  // last visible kv position of rows g and g + 8
#pragma unroll
  for (int i = 0; i < 2; ++i) lim[i] = causal_start >= 0 ? causal_start + (r0 + g + 8 * i) / H : L - 1;

  float m[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
  float o[kMlaVW / 8][4];
#pragma unroll
  for (int dn = 0; dn < kMlaVW / 8; ++dn)
#pragma unroll
    for (int i = 0; i < 4; ++i) o[dn][i] = 0.f;
  for (int jt = 0; jt < ntiles; ++jt) {
    cp_async_wait<kMlaStages - 2>();  // this thread's copies of tile jt have landed
    __syncthreads();                  // everyone's have; every warp is done with tile jt - 1
    if (jt + kMlaStages - 1 < ntiles) issue(jt + kMlaStages - 1);  // into the stage of tile jt - 1
    cp_async_commit();
    const uint16_t* kd = ring + (jt % kMlaStages) * MlaSmem::kTileElems;
    // partial S = Q K^T over this warp's key features (two n8 tiles of positions)
    float sc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
    for (int kk = 0; kk < kMlaKS; ++kk) {
      const int mi = lane >> 3;
      uint32_t b0, b1, b2, b3;
      ldmatrix_x4(b0, b1, b2, b3,
                  kd + ((mi >> 1) * 8 + (lane & 7)) * kMlaRow + (warp * kMlaKS + kk) * 16 + (mi & 1) * 8);
      mma_16816<true>(sc[0], qah[kk], b0, b1);
      mma_16816<true>(sc[0], qal[kk], b0, b1);
      mma_16816<true>(sc[1], qah[kk], b2, b3);
      mma_16816<true>(sc[1], qal[kk], b2, b3);
    }
    // S = the four partial tiles, summed in warp order (the same fragment slots in every warp)
    float* mine = red + (warp * 32 + lane) * 8;
#pragma unroll
    for (int n = 0; n < 2; ++n)
#pragma unroll
      for (int i = 0; i < 4; ++i) mine[n * 4 + i] = sc[n][i];
    __syncthreads();
#pragma unroll
    for (int n = 0; n < 2; ++n)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float s = 0.f;
#pragma unroll
        for (int w = 0; w < kMlaWarps; ++w) s += red[(w * 32 + lane) * 8 + n * 4 + i];
        sc[n][i] = s;
      }
    // scale, mask; element (n, i): row g + 8 (i >> 1), position p0 + 8 n + 2 t + (i & 1)
    const int p0 = k0 + jt * kMlaTile;
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int n = 0; n < 2; ++n)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float x = sc[n][i] * scale;
        const int pos = p0 + 8 * n + 2 * t + (i & 1);
        if (pos >= k1 || pos > lim[i >> 1]) x = -INFINITY;
        sc[n][i] = x;
        mx[i >> 1] = fmaxf(mx[i >> 1], x);
      }
    float mnew[2], alpha[2], rs[2] = {0.f, 0.f};
#pragma unroll
    for (int ri = 0; ri < 2; ++ri) {
      mx[ri] = fmaxf(mx[ri], __shfl_xor_sync(0xffffffffu, mx[ri], 1));
      mx[ri] = fmaxf(mx[ri], __shfl_xor_sync(0xffffffffu, mx[ri], 2));
      mnew[ri] = fmaxf(m[ri], mx[ri]);
      alpha[ri] = mnew[ri] == -INFINITY ? 1.f : expf(m[ri] - mnew[ri]);
    }
#pragma unroll
    for (int n = 0; n < 2; ++n)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int ri = i >> 1;
        const float p = mnew[ri] == -INFINITY ? 0.f : expf(sc[n][i] - mnew[ri]);
        sc[n][i] = p;
        rs[ri] += p;
      }
#pragma unroll
    for (int ri = 0; ri < 2; ++ri) {
      rs[ri] += __shfl_xor_sync(0xffffffffu, rs[ri], 1);
      rs[ri] += __shfl_xor_sync(0xffffffffu, rs[ri], 2);
      l[ri] = l[ri] * alpha[ri] + rs[ri];
      m[ri] = mnew[ri];
    }
#pragma unroll
    for (int dn = 0; dn < kMlaVW / 8; ++dn) {
      o[dn][0] *= alpha[0];
      o[dn][1] *= alpha[0];
      o[dn][2] *= alpha[1];
      o[dn][3] *= alpha[1];
    }
    uint32_t ph[4], pl[4];
    split_bf16x2(sc[0][0], sc[0][1], ph[0], pl[0]);
    split_bf16x2(sc[0][2], sc[0][3], ph[1], pl[1]);
    split_bf16x2(sc[1][0], sc[1][1], ph[2], pl[2]);
    split_bf16x2(sc[1][2], sc[1][3], ph[3], pl[3]);
    // O += P V over this warp's value features (the latent part of the staged rows)
#pragma unroll
    for (int dp = 0; dp < kMlaVW / 16; ++dp) {
      const int mi = lane >> 3;
      uint32_t b0, b1, b2, b3;
      ldmatrix_x4_trans(b0, b1, b2, b3,
                        kd + ((mi & 1) * 8 + (lane & 7)) * kMlaRow + warp * kMlaVW + dp * 16 + (mi >> 1) * 8);
      mma_16816<true>(o[2 * dp], ph, b0, b1);
      mma_16816<true>(o[2 * dp], pl, b0, b1);
      mma_16816<true>(o[2 * dp + 1], ph, b2, b3);
      mma_16816<true>(o[2 * dp + 1], pl, b2, b3);
    }
  }
  // every warp holds the same (m, l) and its own 128 output features of rows g and g + 8
  const size_t rows_total = (size_t)gridDim.y * nrows;  // B * S * H
#pragma unroll
  for (int hi = 0; hi < 2; ++hi) {
    const int r = r0 + g + 8 * hi;
    if (r >= nrows) continue;
    const size_t orow = (size_t)b * nrows + r;
    const float inv = 1.f / fmaxf(l[hi], 1e-30f);
    float* p = splits > 1 ? part + ((size_t)split * rows_total + orow) * (kMlaR + 2) : nullptr;
    if (p && warp == 0 && t == 0) {
      p[0] = m[hi];
      p[1] = l[hi];
    }
#pragma unroll
    for (int dn = 0; dn < kMlaVW / 8; ++dn) {
      const int f = warp * kMlaVW + dn * 8 + 2 * t;
      const float v0 = o[dn][2 * hi], v1 = o[dn][2 * hi + 1];
      if (p) {
        p[2 + f] = v0;
        p[3 + f] = v1;
      } else if constexpr (OUT_BF16) {
        static_cast<__nv_bfloat16*>(out)[orow * kMlaR + f] = __float2bfloat16_rn(v0 * inv);
        static_cast<__nv_bfloat16*>(out)[orow * kMlaR + f + 1] = __float2bfloat16_rn(v1 * inv);
      } else {
        static_cast<float*>(out)[orow * kMlaR + f] = v0 * inv;
        static_cast<float*>(out)[orow * kMlaR + f + 1] = v1 * inv;
      }
    }
  }
}

template <bool OUT_BF16>
__global__ void __launch_bounds__(kMlaWarps * 32) mla_attn_kernel(
    const float* __restrict__ q, const uint16_t* __restrict__ kv, int H, int S, int L, int causal_start, float scale,
    int splits, int tiles_per_split, void* __restrict__ out, float* __restrict__ part) {
  mla_attn_body<OUT_BF16, false>(q, kv, H, S, L, causal_start, scale, splits, tiles_per_split, out, part, nullptr,
                                 nullptr, 0, 0);
}

template <bool OUT_BF16>
__global__ void __launch_bounds__(kMlaWarps * 32) mla_attn_pool_kernel(
    const float* __restrict__ q, const uint16_t* __restrict__ kv, int H, int S, int L, float scale, int splits,
    int tiles_per_split, void* __restrict__ out, float* __restrict__ part, const int* __restrict__ slots,
    const int* __restrict__ starts, long long slot_stride, int num_slots) {
  mla_attn_body<OUT_BF16, true>(q, kv, H, S, L, 0, scale, splits, tiles_per_split, out, part, slots, starts,
                                slot_stride, num_slots);
}

// RMSNorm of one row per CTA (128 threads, any dim).
template <bool IN_BF16, bool OUT_BF16>
__global__ void __launch_bounds__(128) rms_norm_kernel(const void* __restrict__ x, const float* __restrict__ w,
                                                       int dim, float eps, void* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  __shared__ float red[4];
  const int row = blockIdx.x, tid = threadIdx.x;
  auto load = [&](int i) -> float {
    if constexpr (IN_BF16) return bf16_to_f32(static_cast<const uint16_t*>(x)[(size_t)row * dim + i]);
    else return static_cast<const float*>(x)[(size_t)row * dim + i];
  };
  float ss = 0.f;
  for (int i = tid; i < dim; i += blockDim.x) {
    const float a = load(i);
    ss = fmaf(a, a, ss);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((tid & 31) == 0) red[tid >> 5] = ss;
  __syncthreads();
  const float tot = (red[0] + red[1]) + (red[2] + red[3]);
  const float r = 1.f / sqrtf(tot / (float)dim + eps);
  for (int i = tid; i < dim; i += blockDim.x) {
    float y = load(i) * r;
    if (w) y *= w[i];
    if constexpr (OUT_BF16) static_cast<__nv_bfloat16*>(out)[(size_t)row * dim + i] = __float2bfloat16_rn(y);
    else static_cast<float*>(out)[(size_t)row * dim + i] = y;
  }
}

// RoPE, half rotation (ccut/blocks/rope.py:130-175): for the pair (i, i + d/2) of a row
// (b, head, s), f = positions[b, s] * inv_freq[i] (fp32), out_i = x_i cos f - x_{i+d/2} sin f,
// out_{i+d/2} = x_{i+d/2} cos f + x_i sin f, with x first multiplied by `scale` (the
// attention factor the reference applies to q).  Products are rounded before the sums, as
// in the reference's numpy expression.
template <bool IN_BF16, bool OUT_BF16>
__global__ void __launch_bounds__(256) rope_kernel(const void* __restrict__ x, int heads, int S, int half,
                                                   const float* __restrict__ inv_freq,
                                                   const int32_t* __restrict__ positions, float scale,
                                                   long long n_pairs, void* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  for (long long idx = blockIdx.x * (long long)blockDim.x + threadIdx.x; idx < n_pairs;
       idx += (long long)gridDim.x * blockDim.x) {
    const int i = (int)(idx % half);
    const long long row = idx / half;
    const int s = (int)(row % S);
    const long long b = row / S / heads;
    const float f = __fmul_rn((float)positions[b * S + s], inv_freq[i]);
    const float c = cosf(f), sn = sinf(f);
    const size_t o1 = (size_t)row * (2 * half) + i, o2 = o1 + half;
    float x1, x2;
    if constexpr (IN_BF16) {
      x1 = bf16_to_f32(static_cast<const uint16_t*>(x)[o1]);
      x2 = bf16_to_f32(static_cast<const uint16_t*>(x)[o2]);
    } else {
      x1 = static_cast<const float*>(x)[o1];
      x2 = static_cast<const float*>(x)[o2];
    }
    x1 = __fmul_rn(x1, scale);
    x2 = __fmul_rn(x2, scale);
    const float y1 = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, sn));
    const float y2 = __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, sn));
    if constexpr (OUT_BF16) {
      static_cast<__nv_bfloat16*>(out)[o1] = __float2bfloat16_rn(y1);
      static_cast<__nv_bfloat16*>(out)[o2] = __float2bfloat16_rn(y2);
    } else {
      static_cast<float*>(out)[o1] = y1;
      static_cast<float*>(out)[o2] = y2;
    }
  }
}

// kv splits: enough CTAs to cover the SMs twice, at least one 64-position tile per split.
// kv splits of the MLA kernel: enough CTAs to cover the SMs twice, at least one 64-position
// stretch per split.
static int mla_splits(int B, int H, int S, int L) {
  const long base = (long)(((long)S * H + kTcRows - 1) / kTcRows) * B;
  const int tiles = (L + kAttnTile - 1) / kAttnTile;
  long sp = base > 0 ? (2L * 148 + base - 1) / base : 1;
  if (sp > tiles) sp = tiles;
  if (sp > 64) sp = 64;
  return sp < 1 ? 1 : (int)sp;
}

static int attn_splits(int B, int Hq, int Hkv, int S, int L) {
  const int G = Hq / Hkv;
  const long base = (long)((G * S + kTcRows - 1) / kTcRows) * B * Hkv;
  const int tiles = (L + kAttnTile - 1) / kAttnTile;
  long sp = (2L * 148 + base - 1) / base;
  if (sp > tiles) sp = tiles;
  if (sp > 64) sp = 64;
  return sp < 1 ? 1 : (int)sp;
}

static bool attn_shape_ok(int B, int Hq, int Hkv, int S, int L, int D) {
  return B >= 0 && Hq > 0 && Hkv > 0 && Hq % Hkv == 0 && S >= 0 && L >= 0 && (D == 64 || D == 128);
}

}  // namespace ccut

using namespace ccut;

extern "C" {

size_t ccut_gqa_attention_workspace_bytes(int batch, int heads, int kv_heads, int seq, int kv_len, int head_dim) {
  if (!attn_shape_ok(batch, heads, kv_heads, seq, kv_len, head_dim)) return 0;
  const int sp = attn_splits(batch, heads, kv_heads, seq, kv_len);
  if (sp <= 1) return 256;
  return 256 + (size_t)sp * batch * heads * seq * (head_dim + 2) * sizeof(float);
}

int ccut_gqa_attention(const uint16_t* q, const uint16_t* k, const uint16_t* v, int batch, int heads, int kv_heads,
                       int seq, int kv_len, int head_dim, int causal_start, float scale, float softcap, void* out,
                       int out_dtype, void* workspace, size_t ws_bytes, ccut_stream_t stream) {
  PdlScope pdl_scope((long)batch * seq);
  if (head_dim != 64 && head_dim != 128) return CCUT_ERR_UNSUPPORTED;
  if (!attn_shape_ok(batch, heads, kv_heads, seq, kv_len, head_dim)) return CCUT_ERR_INVALID;
  if (out_dtype != CCUT_OUT_BF16 && out_dtype != CCUT_OUT_F32) return CCUT_ERR_INVALID;
  if (batch == 0 || seq == 0) return CCUT_OK;
  if (!q || !out || (kv_len > 0 && (!k || !v))) return CCUT_ERR_INVALID;
  if ((size_t)batch * kv_heads > 65535) return CCUT_ERR_UNSUPPORTED;
  const size_t need = ccut_gqa_attention_workspace_bytes(batch, heads, kv_heads, seq, kv_len, head_dim);
  const int sp = attn_splits(batch, heads, kv_heads, seq, kv_len);
  if (sp > 1 && (!workspace || ws_bytes < need)) return CCUT_ERR_WORKSPACE;
  if (!(scale > 0.f)) scale = 1.f / sqrtf((float)head_dim);
  const int G = heads / kv_heads;
  const int tiles = (kv_len + kAttnTile - 1) / kAttnTile;
  const int tps = sp > 0 ? (tiles + sp - 1) / sp : 1;
  const dim3 grid((G * seq + kTcRows - 1) / kTcRows, batch * kv_heads, sp);
  float* part = sp > 1 ? reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + 256) : nullptr;
  const bool ob = out_dtype == CCUT_OUT_BF16;
  int rc;
  if (head_dim == 128) {
    auto kern = ob ? gqa_attn_kernel<128, true> : gqa_attn_kernel<128, false>;
    constexpr size_t smem = TcAttnSmem<128>::kBytes;
    static std::atomic<uint64_t> smem_set[2];  // per output type: devices with the limit raised
    rc = ensure_smem_limit(kern, smem, smem_set[ob]);
    if (rc) return rc;
    rc = launch_k(kern, grid, dim3(kTcWarps * 32), smem, stream, q, k, v, heads, kv_heads, seq, kv_len, causal_start,
                  scale, softcap, sp, tps, out, part);
  } else {
    auto kern = ob ? gqa_attn_kernel<64, true> : gqa_attn_kernel<64, false>;
    constexpr size_t smem = TcAttnSmem<64>::kBytes;
    static std::atomic<uint64_t> smem_set[2];
    rc = ensure_smem_limit(kern, smem, smem_set[ob]);
    if (rc) return rc;
    rc = launch_k(kern, grid, dim3(kTcWarps * 32), smem, stream, q, k, v, heads, kv_heads, seq, kv_len, causal_start,
                  scale, softcap, sp, tps, out, part);
  }
  if (rc || sp == 1) return rc;
  const int rows = batch * heads * seq;
  const dim3 g2((rows + 7) / 8);
  if (head_dim == 128)
    return launch_k(ob ? gqa_combine_kernel<128, true> : gqa_combine_kernel<128, false>, g2, dim3(256), 0, stream,
                    (const float*)part, rows, sp, out);
  return launch_k(ob ? gqa_combine_kernel<64, true> : gqa_combine_kernel<64, false>, g2, dim3(256), 0, stream,
                  (const float*)part, rows, sp, out);
}

int ccut_gqa_attention_pool(const uint16_t* q, const uint16_t* k_pool, const uint16_t* v_pool, const int32_t* slots,
                            const int32_t* starts, int batch, int heads, int kv_heads, int seq, int max_len,
                            int head_dim, long long slot_stride, int num_slots, float scale, float softcap, void* out,
                            int out_dtype, void* workspace, size_t ws_bytes, ccut_stream_t stream) {
  PdlScope pdl_scope((long)batch * seq);
  if (head_dim != 64 && head_dim != 128) return CCUT_ERR_UNSUPPORTED;
  if (!attn_shape_ok(batch, heads, kv_heads, seq, max_len, head_dim) || num_slots < 0) return CCUT_ERR_INVALID;
  if (out_dtype != CCUT_OUT_BF16 && out_dtype != CCUT_OUT_F32) return CCUT_ERR_INVALID;
  if (slot_stride < (long long)kv_heads * max_len * head_dim || slot_stride % 8) return CCUT_ERR_INVALID;
  if (batch == 0 || seq == 0) return CCUT_OK;
  if (!q || !out || !slots || !starts || (max_len > 0 && num_slots > 0 && (!k_pool || !v_pool)))
    return CCUT_ERR_INVALID;
  if ((size_t)batch * kv_heads > 65535) return CCUT_ERR_UNSUPPORTED;
  const size_t need = ccut_gqa_attention_workspace_bytes(batch, heads, kv_heads, seq, max_len, head_dim);
  const int sp = attn_splits(batch, heads, kv_heads, seq, max_len);
  if (sp > 1 && (!workspace || ws_bytes < need)) return CCUT_ERR_WORKSPACE;
  if (!(scale > 0.f)) scale = 1.f / sqrtf((float)head_dim);
  const int G = heads / kv_heads;
  const int tiles = (max_len + kAttnTile - 1) / kAttnTile;
  const int tps = sp > 0 ? (tiles + sp - 1) / sp : 1;
  const dim3 grid((G * seq + kTcRows - 1) / kTcRows, batch * kv_heads, sp);
  float* part = sp > 1 ? reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + 256) : nullptr;
  const bool ob = out_dtype == CCUT_OUT_BF16;
  const int* sl = reinterpret_cast<const int*>(slots);
  const int* st = reinterpret_cast<const int*>(starts);
  int rc;
  if (head_dim == 128) {
    auto kern = ob ? gqa_attn_pool_kernel<128, true> : gqa_attn_pool_kernel<128, false>;
    constexpr size_t smem = TcAttnSmem<128>::kBytes;
    static std::atomic<uint64_t> smem_set[2];  // per output type: devices with the limit raised
    rc = ensure_smem_limit(kern, smem, smem_set[ob]);
    if (rc) return rc;
    rc = launch_k(kern, grid, dim3(kTcWarps * 32), smem, stream, q, k_pool, v_pool, heads, kv_heads, seq, max_len,
                  scale, softcap, sp, tps, out, part, sl, st, slot_stride, num_slots);
  } else {
    auto kern = ob ? gqa_attn_pool_kernel<64, true> : gqa_attn_pool_kernel<64, false>;
    constexpr size_t smem = TcAttnSmem<64>::kBytes;
    static std::atomic<uint64_t> smem_set[2];
    rc = ensure_smem_limit(kern, smem, smem_set[ob]);
    if (rc) return rc;
    rc = launch_k(kern, grid, dim3(kTcWarps * 32), smem, stream, q, k_pool, v_pool, heads, kv_heads, seq, max_len,
                  scale, softcap, sp, tps, out, part, sl, st, slot_stride, num_slots);
  }
  if (rc || sp == 1) return rc;
  const int rows = batch * heads * seq;
  const dim3 g2((rows + 7) / 8);
  if (head_dim == 128)
    return launch_k(ob ? gqa_combine_kernel<128, true> : gqa_combine_kernel<128, false>, g2, dim3(256), 0, stream,
                    (const float*)part, rows, sp, out);
  return launch_k(ob ? gqa_combine_kernel<64, true> : gqa_combine_kernel<64, false>, g2, dim3(256), 0, stream,
                  (const float*)part, rows, sp, out);
}

size_t ccut_mla_attention_workspace_bytes(int batch, int heads, int seq, int kv_len) {
  if (batch < 0 || heads <= 0 || seq < 0 || kv_len < 0) return 0;
  const int sp = mla_splits(batch, heads, seq, kv_len);
  if (sp <= 1) return 256;
  return 256 + (size_t)sp * batch * heads * seq * (kMlaR + 2) * sizeof(float);
}

int ccut_mla_attention(const float* q, const uint16_t* kv, int batch, int heads, int seq, int kv_len, int rank,
                       int rope_dim, int causal_start, float scale, void* out, int out_dtype, void* workspace,
                       size_t ws_bytes, ccut_stream_t stream) {
  PdlScope pdl_scope((long)batch * seq);
  if (rank != kMlaR || rope_dim != kMlaP) return CCUT_ERR_UNSUPPORTED;
  if (batch < 0 || heads <= 0 || seq < 0 || kv_len < 0 || !(scale > 0.f)) return CCUT_ERR_INVALID;
  if (out_dtype != CCUT_OUT_BF16 && out_dtype != CCUT_OUT_F32) return CCUT_ERR_INVALID;
  if (batch == 0 || seq == 0) return CCUT_OK;
  if (!q || !out || (kv_len > 0 && !kv)) return CCUT_ERR_INVALID;
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(kv)) % 16) return CCUT_ERR_INVALID;
  if (batch > 65535 || (long)seq * heads > 2147483647L - kTcRows) return CCUT_ERR_UNSUPPORTED;
  const int sp = mla_splits(batch, heads, seq, kv_len);
  if (sp > 1 && (!workspace || ws_bytes < ccut_mla_attention_workspace_bytes(batch, heads, seq, kv_len)))
    return CCUT_ERR_WORKSPACE;
  const int nrows = seq * heads;
  const int tiles = (kv_len + kMlaTile - 1) / kMlaTile;
  const int tps = (tiles + sp - 1) / sp;
  const dim3 grid((nrows + kTcRows - 1) / kTcRows, batch, sp);
  float* part = sp > 1 ? reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + 256) : nullptr;
  const bool ob = out_dtype == CCUT_OUT_BF16;
  auto kern = ob ? mla_attn_kernel<true> : mla_attn_kernel<false>;
  static std::atomic<uint64_t> smem_set[2];  // per output type: devices with the limit raised
  int rc = ensure_smem_limit(kern, MlaSmem::kBytes, smem_set[ob]);
  if (rc) return rc;
  rc = launch_k(kern, grid, dim3(kMlaWarps * 32), MlaSmem::kBytes, stream, q, kv, heads, seq, kv_len, causal_start,
                scale, sp, tps, out, part);
  if (rc || sp == 1) return rc;
  const int rows = batch * nrows;
  return launch_k(ob ? gqa_combine_kernel<kMlaR, true> : gqa_combine_kernel<kMlaR, false>, dim3((rows + 7) / 8),
                  dim3(256), 0, stream, (const float*)part, rows, sp, out);
}

int ccut_mla_attention_pool(const float* q, const uint16_t* kv_pool, const int32_t* slots, const int32_t* starts,
                            int batch, int heads, int seq, int max_len, int rank, int rope_dim, long long slot_stride,
                            int num_slots, float scale, void* out, int out_dtype, void* workspace, size_t ws_bytes,
                            ccut_stream_t stream) {
  PdlScope pdl_scope((long)batch * seq);
  if (rank != kMlaR || rope_dim != kMlaP) return CCUT_ERR_UNSUPPORTED;
  if (batch < 0 || heads <= 0 || seq < 0 || max_len < 0 || num_slots < 0 || !(scale > 0.f)) return CCUT_ERR_INVALID;
  if (out_dtype != CCUT_OUT_BF16 && out_dtype != CCUT_OUT_F32) return CCUT_ERR_INVALID;
  if (slot_stride < (long long)max_len * kMlaK || slot_stride % 8) return CCUT_ERR_INVALID;
  if (batch == 0 || seq == 0) return CCUT_OK;
  if (!q || !out || !slots || !starts || (max_len > 0 && num_slots > 0 && !kv_pool)) return CCUT_ERR_INVALID;
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(kv_pool)) % 16) return CCUT_ERR_INVALID;
  if (batch > 65535 || (long)seq * heads > 2147483647L - kTcRows) return CCUT_ERR_UNSUPPORTED;
  const int sp = mla_splits(batch, heads, seq, max_len);
  if (sp > 1 && (!workspace || ws_bytes < ccut_mla_attention_workspace_bytes(batch, heads, seq, max_len)))
    return CCUT_ERR_WORKSPACE;
  const int nrows = seq * heads;
  const int tiles = (max_len + kMlaTile - 1) / kMlaTile;
  const int tps = (tiles + sp - 1) / sp;
  const dim3 grid((nrows + kTcRows - 1) / kTcRows, batch, sp);
  float* part = sp > 1 ? reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + 256) : nullptr;
  const bool ob = out_dtype == CCUT_OUT_BF16;
  auto kern = ob ? mla_attn_pool_kernel<true> : mla_attn_pool_kernel<false>;
  static std::atomic<uint64_t> smem_set[2];  // per output type: devices with the limit raised
  int rc = ensure_smem_limit(kern, MlaSmem::kBytes, smem_set[ob]);
  if (rc) return rc;
  rc = launch_k(kern, grid, dim3(kMlaWarps * 32), MlaSmem::kBytes, stream, q, kv_pool, heads, seq, max_len, scale, sp,
                tps, out, part, reinterpret_cast<const int*>(slots), reinterpret_cast<const int*>(starts), slot_stride,
                num_slots);
  if (rc || sp == 1) return rc;
  const int rows = batch * nrows;
  return launch_k(ob ? gqa_combine_kernel<kMlaR, true> : gqa_combine_kernel<kMlaR, false>, dim3((rows + 7) / 8),
                  dim3(256), 0, stream, (const float*)part, rows, sp, out);
}

int ccut_apply_rope(const void* x, int x_dtype, int batch, int heads, int seq, int head_dim, const float* inv_freq,
                    const int32_t* positions, float scale, void* out, int out_dtype, ccut_stream_t stream) {
  PdlScope pdl_scope((long)batch * seq);
  if (batch < 0 || heads <= 0 || seq < 0 || head_dim <= 0 || head_dim % 2) return CCUT_ERR_INVALID;
  if ((x_dtype != CCUT_OUT_BF16 && x_dtype != CCUT_OUT_F32) || (out_dtype != CCUT_OUT_BF16 && out_dtype != CCUT_OUT_F32))
    return CCUT_ERR_INVALID;
  const long long n_pairs = (long long)batch * heads * seq * (head_dim / 2);
  if (n_pairs == 0) return CCUT_OK;
  if (!x || !inv_freq || !positions || !out) return CCUT_ERR_INVALID;
  long long blocks = (n_pairs + 255) / 256;
  if (blocks > 148 * 32) blocks = 148 * 32;
  const bool ib = x_dtype == CCUT_OUT_BF16, ob = out_dtype == CCUT_OUT_BF16;
  auto kern = ib ? (ob ? rope_kernel<true, true> : rope_kernel<true, false>)
                 : (ob ? rope_kernel<false, true> : rope_kernel<false, false>);
  return launch_k(kern, dim3((unsigned)blocks), dim3(256), 0, stream, x, heads, seq, head_dim / 2, inv_freq,
                  positions, scale, n_pairs, out);
}

int ccut_rms_norm(const void* x, int x_dtype, const float* weight, int rows, int dim, float eps, void* out,
                  int out_dtype, ccut_stream_t stream) {
  PdlScope pdl_scope(rows);
  if (rows < 0 || dim <= 0 || !(eps >= 0.f)) return CCUT_ERR_INVALID;
  if ((x_dtype != CCUT_OUT_BF16 && x_dtype != CCUT_OUT_F32) || (out_dtype != CCUT_OUT_BF16 && out_dtype != CCUT_OUT_F32))
    return CCUT_ERR_INVALID;
  if (rows == 0) return CCUT_OK;
  if (!x || !out) return CCUT_ERR_INVALID;
  if (rows > 2147483647) return CCUT_ERR_UNSUPPORTED;
  const bool ib = x_dtype == CCUT_OUT_BF16, ob = out_dtype == CCUT_OUT_BF16;
  auto kern = ib ? (ob ? rms_norm_kernel<true, true> : rms_norm_kernel<true, false>)
                 : (ob ? rms_norm_kernel<false, true> : rms_norm_kernel<false, false>);
  return launch_k(kern, dim3(rows), dim3(128), 0, stream, x, weight, dim, eps, out);
}

}  // extern "C"
