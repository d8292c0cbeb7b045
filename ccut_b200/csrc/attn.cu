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
// Work: a CTA takes 8 query rows of one (batch, kv head) -- the query heads that share the
// kv head, row r = (s, g) with s = r / G, g = r % G -- and one split of the kv range.  K and
// V tiles of 64 positions are staged in shared memory (K transposed, so that lane l reads
// positions 2l, 2l+1 of one d without bank conflicts); each warp owns one query row and
// keeps an online softmax (running max m, sum l, fp32 accumulator over its D/32 output
// dims).  With one split the CTA writes o = acc / max(l, 1e-30); with several it writes
// (m, l, acc) and gqa_combine_kernel merges the splits.  Bound: HBM (K and V read once per
// (batch, kv head, split); query rows of a kv head share them).
//
// RMSNorm: y = x * (mean(x^2) + eps)^-1/2 * w per row in fp32 (ccut/blocks/norm.py:14-26).
#include <math.h>

#include "host.cuh"

namespace ccut {

constexpr int kAttnRows = 8;   // query rows (warps) per CTA
constexpr int kAttnTile = 64;  // kv positions per staged tile

__device__ __forceinline__ float bf16_to_f32(uint16_t b) { return __uint_as_float((uint32_t)b << 16); }

template <int D, bool OUT_BF16>
__global__ void __launch_bounds__(256) gqa_attn_kernel(const uint16_t* __restrict__ q, const uint16_t* __restrict__ k,
                                                       const uint16_t* __restrict__ v, int Hq, int Hkv, int S, int L,
                                                       int causal_start, float scale, float softcap, int splits,
                                                       int tiles_per_split, void* __restrict__ out,
                                                       float* __restrict__ part) {
  pdl_wait();
  pdl_trigger();
  constexpr int DL = D / 32;  // output dims per lane
  // K transposed, rows padded to 66 elements: the transposing stores then conflict 4-way
  // instead of 16-way, and the per-lane score reads (one 32-bit word per lane) stay
  // conflict-free
  __shared__ __align__(16) uint16_t kT[D][kAttnTile + 2];
  __shared__ __align__(16) uint16_t vt[kAttnTile][D];
  __shared__ __align__(16) float qs[kAttnRows][D];
  __shared__ float ps[kAttnRows][kAttnTile];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = Hq / Hkv;
  const int bh = blockIdx.y;  // b * Hkv + kvh
  const int b = bh / Hkv, kvh = bh % Hkv;
  const int r = blockIdx.x * kAttnRows + warp;  // query row within (b, kvh)
  const bool row_ok = r < G * S;
  const int s = row_ok ? r / G : 0, h = kvh * G + (row_ok ? r % G : 0);
  const int split = blockIdx.z;
  const int k0 = split * tiles_per_split * kAttnTile;
  int k1 = min(L, k0 + tiles_per_split * kAttnTile);
  // causal: the CTA's last row sees up to causal_start + s_last
  if (causal_start >= 0) {
    const int r_last = min(G * S, (int)(blockIdx.x + 1) * kAttnRows) - 1;
    k1 = min(k1, causal_start + r_last / G + 1);
  }
  const int lim = causal_start >= 0 ? causal_start + s : L - 1;  // last visible position of this row
  const uint16_t* kb = k + (size_t)bh * L * D;
  const uint16_t* vb = v + (size_t)bh * L * D;
  if (row_ok) {
    const uint16_t* qr = q + (((size_t)b * Hq + h) * S + s) * D;
    for (int d = lane; d < D; d += 32) qs[warp][d] = bf16_to_f32(qr[d]);
  }
  float m = -INFINITY, l = 0.f, acc[DL];
#pragma unroll
  for (int j = 0; j < DL; ++j) acc[j] = 0.f;

  for (int t0 = k0; t0 < k1; t0 += kAttnTile) {
    __syncthreads();  // previous tile consumed (and qs written, first time)
    constexpr int kChunks = kAttnTile * D / 8;  // 16-byte chunks per tile
    for (int c = threadIdx.x; c < kChunks; c += blockDim.x) {
      const int p = c / (D / 8), dc = (c % (D / 8)) * 8;
      uint4 kk = make_uint4(0, 0, 0, 0), vv = make_uint4(0, 0, 0, 0);
      if (t0 + p < k1) {
        kk = *reinterpret_cast<const uint4*>(kb + (size_t)(t0 + p) * D + dc);
        vv = *reinterpret_cast<const uint4*>(vb + (size_t)(t0 + p) * D + dc);
      }
      *reinterpret_cast<uint4*>(&vt[p][dc]) = vv;
      const uint32_t w4[4] = {kk.x, kk.y, kk.z, kk.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        kT[dc + 2 * j][p] = (uint16_t)(w4[j] & 0xffffu);
        kT[dc + 2 * j + 1][p] = (uint16_t)(w4[j] >> 16);
      }
    }
    __syncthreads();
    if (!row_ok) continue;
    // scores of positions p0 = 2 lane, p0 + 1
    float s0 = 0.f, s1 = 0.f;
#pragma unroll 8
    for (int d = 0; d < D; ++d) {
      const float qd = qs[warp][d];
      const uint32_t kk = *reinterpret_cast<const uint32_t*>(&kT[d][2 * lane]);
      s0 = fmaf(qd, __uint_as_float(kk << 16), s0);
      s1 = fmaf(qd, __uint_as_float(kk & 0xffff0000u), s1);
    }
    s0 *= scale;
    s1 *= scale;
    if (softcap > 0.f) {
      s0 = tanhf(s0 / softcap) * softcap;
      s1 = tanhf(s1 / softcap) * softcap;
    }
    const int pos0 = t0 + 2 * lane;
    if (pos0 >= k1 || pos0 > lim) s0 = -INFINITY;
    if (pos0 + 1 >= k1 || pos0 + 1 > lim) s1 = -INFINITY;
    float mt = fmaxf(s0, s1);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, o));
    const float m_new = fmaxf(m, mt);
    float p0 = 0.f, p1 = 0.f, alpha = 1.f;
    if (m_new > -INFINITY) {
      alpha = expf(m - m_new);  // 0 while nothing was visible (m = -inf)
      p0 = expf(s0 - m_new);
      p1 = expf(s1 - m_new);
    }
    float ts = p0 + p1;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ts += __shfl_xor_sync(0xffffffffu, ts, o);
    l = l * alpha + ts;
    m = m_new;
    ps[warp][2 * lane] = p0;
    ps[warp][2 * lane + 1] = p1;
    __syncwarp();
#pragma unroll
    for (int j = 0; j < DL; ++j) acc[j] *= alpha;
    const int npos = min(kAttnTile, k1 - t0);
    for (int p = 0; p < npos; ++p) {
      const float pp = ps[warp][p];
      if constexpr (DL == 4) {
        const uint2 vv = *reinterpret_cast<const uint2*>(&vt[p][lane * 4]);
        acc[0] = fmaf(pp, __uint_as_float(vv.x << 16), acc[0]);
        acc[1] = fmaf(pp, __uint_as_float(vv.x & 0xffff0000u), acc[1]);
        acc[2] = fmaf(pp, __uint_as_float(vv.y << 16), acc[2]);
        acc[3] = fmaf(pp, __uint_as_float(vv.y & 0xffff0000u), acc[3]);
      } else {
        const uint32_t vv = *reinterpret_cast<const uint32_t*>(&vt[p][lane * 2]);
        acc[0] = fmaf(pp, __uint_as_float(vv << 16), acc[0]);
        acc[1] = fmaf(pp, __uint_as_float(vv & 0xffff0000u), acc[1]);
      }
    }
    __syncwarp();
  }
  if (!row_ok) return;
  const size_t orow = ((size_t)b * Hq + h) * S + s;
  if (splits == 1) {
    const float inv = 1.f / fmaxf(l, 1e-30f);
#pragma unroll
    for (int j = 0; j < DL; ++j) {
      const float o = acc[j] * inv;
      const size_t idx = orow * D + lane * DL + j;
      if constexpr (OUT_BF16) static_cast<__nv_bfloat16*>(out)[idx] = __float2bfloat16_rn(o);
      else static_cast<float*>(out)[idx] = o;
    }
  } else {
    const size_t rows_total = (size_t)gridDim.y / Hkv * Hq * S;  // B * Hq * S
    float* p = part + ((size_t)split * rows_total + orow) * (D + 2);
    if (lane == 0) {
      p[0] = m;
      p[1] = l;
    }
#pragma unroll
    for (int j = 0; j < DL; ++j) p[2 + lane * DL + j] = acc[j];
  }
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

// RMSNorm of one row per CTA (128 threads, dim % 8 == 0).
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

// kv splits: enough CTAs to cover the SMs twice, at least one 64-position tile per split.
static int attn_splits(int B, int Hq, int Hkv, int S, int L) {
  const int G = Hq / Hkv;
  const long base = (long)((G * S + kAttnRows - 1) / kAttnRows) * B * Hkv;
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
  const dim3 grid((G * seq + kAttnRows - 1) / kAttnRows, batch * kv_heads, sp);
  float* part = sp > 1 ? reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + 256) : nullptr;
  const bool ob = out_dtype == CCUT_OUT_BF16;
  int rc;
  if (head_dim == 128)
    rc = launch_k(ob ? gqa_attn_kernel<128, true> : gqa_attn_kernel<128, false>, grid, dim3(256), 0, stream, q, k, v,
                  heads, kv_heads, seq, kv_len, causal_start, scale, softcap, sp, tps, out, part);
  else
    rc = launch_k(ob ? gqa_attn_kernel<64, true> : gqa_attn_kernel<64, false>, grid, dim3(256), 0, stream, q, k, v,
                  heads, kv_heads, seq, kv_len, causal_start, scale, softcap, sp, tps, out, part);
  if (rc || sp == 1) return rc;
  const int rows = batch * heads * seq;
  const dim3 g2((rows + 7) / 8);
  if (head_dim == 128)
    return launch_k(ob ? gqa_combine_kernel<128, true> : gqa_combine_kernel<128, false>, g2, dim3(256), 0, stream,
                    (const float*)part, rows, sp, out);
  return launch_k(ob ? gqa_combine_kernel<64, true> : gqa_combine_kernel<64, false>, g2, dim3(256), 0, stream,
                  (const float*)part, rows, sp, out);
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
