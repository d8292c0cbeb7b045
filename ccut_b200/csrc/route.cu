// route.cu -- router logits, top-k and token permutation.
//
//   logits[t, e] = sum_h x[t, h] * router[e, h]   fp32 (ccut/models/generic.py:361)
//   top-k per token, three modes                  (ccut/blocks/moe.py:46-89 + grouped sigmoid)
//   stable counting sort of (token, slot) pairs by expert (ccut/models/generic.py:367-371)
//
// The logits GEMV splits H across CTAs so that a decode batch still spreads over the SMs;
// the partial sums are added in a fixed order by the top-k kernel, so the routing is
// deterministic run to run.
#include <math.h>

#include <algorithm>

#include "launch.cuh"
#include "layout.cuh"

namespace ccut {

constexpr int kRtTok = 64;   // tokens per logits CTA
constexpr int kRtExp = 64;   // experts per logits CTA
constexpr int kRtH = 64;     // h per shared-memory chunk
constexpr int kRtPitch = 72; // bf16 per staged row (64 + 8): conflict-free ldmatrix rows
constexpr int kRtTiledMinT = 256;  // from this batch size on: split once, then the pipelined GEMM

// Number of H splits: enough CTAs to cover the SMs at small T, one split at large T.
int route_hsplit(int T, int E, int H) {
  const int chunks = H / kRtH;
  const int ctas = ((T + kRtTok - 1) / kRtTok) * ((E + kRtExp - 1) / kRtExp);
  int hs = (296 + ctas - 1) / ctas;
  if (hs > chunks) hs = chunks;
  if (hs < 1) hs = 1;
  while (chunks % hs) --hs;
  return hs;
}

// fp32 scratch of launch_route: the H-split partial logits, then (T >= kRtTiledMinT) the router's
// three bf16 split planes, 16-byte aligned.
size_t route_scratch_floats(int T, int E, int H) {
  size_t n = (size_t)route_hsplit(T, E, H) * T * E;
  if (T >= kRtTiledMinT) n = (n + 3) / 4 * 4 + ((size_t)3 * E * H + 1) / 2;
  return n;
}

// An amount of that scratch that serves every batch of at most T_cap tokens: the split count
// hs <= 296 / ctas + 1 with ctas >= T / 64 tiles gives hs * T <= 296 * 64 + T, and hs <= H / 64.
size_t route_scratch_floats_upto(int T_cap, int E, int H) {
  const size_t ht = std::min((size_t)(H / kRtH) * T_cap, (size_t)296 * kRtTok + T_cap);
  size_t n = ht * E;
  if (T_cap >= kRtTiledMinT) n = (n + 3) / 4 * 4 + ((size_t)3 * E * H + 1) / 2;
  return n;
}

// fp32 -> (hi, mid, lo) bf16 with hi + mid + lo == w exactly: each part keeps the next 8
// significant bits of the remainder (bf16 has fp32's exponent range).
__device__ __forceinline__ void split3_bf16(float w, uint16_t& hi, uint16_t& mid, uint16_t& lo) {
  const __nv_bfloat16 h = __float2bfloat16_rn(w);
  const float r1 = w - __bfloat162float(h);
  const __nv_bfloat16 m = __float2bfloat16_rn(r1);
  const __nv_bfloat16 l = __float2bfloat16_rn(r1 - __bfloat162float(m));
  hi = __bfloat16_as_ushort(h);
  mid = __bfloat16_as_ushort(m);
  lo = __bfloat16_as_ushort(l);
}

// part[hs][t][e] = sum over this split's h of x[t, h] * router[e, h] (fp32) on the tensor
// cores: the bf16 activations are exact operands and each fp32 router weight is the exact sum
// of three bf16 parts, so every product is exact and only the fp32 accumulation rounds, as in
// an fp32 GEMM.  CTA tile 64 tokens x 64 experts; warp w owns tokens 16 (w & 3) .. + 15 and
// experts 32 (w >> 2) .. + 31 (four m16n8k16 column tiles, three MMAs each per 16-h step).
// Also zeroes counts[E] and writes x16 (f16 copy of x) when requested.
__global__ void __launch_bounds__(256) route_logits_kernel(const uint16_t* __restrict__ x,
                                                           const float* __restrict__ router, int T, int H, int E,
                                                           int hsplit, float* __restrict__ part,
                                                           int* __restrict__ counts, uint16_t* __restrict__ x16) {
  pdl_wait();
  pdl_trigger();
  __shared__ __align__(16) uint16_t xs[kRtTok * kRtPitch];     // [token][h]
  __shared__ __align__(16) uint16_t ws[3][kRtExp * kRtPitch];  // [part][expert][h]
  const int t0 = blockIdx.x * kRtTok, e0 = blockIdx.y * kRtExp, hs = blockIdx.z;
  const int hlen = H / hsplit, hbeg = hs * hlen;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (counts && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0)
    for (int e = tid; e < E; e += blockDim.x) counts[e] = 0;
  const int tg = warp & 3, eh = warp >> 2;
  float acc[4][4];
#pragma unroll
  for (int j = 0; j < 4; ++j)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[j][i] = 0.f;
  for (int h0 = hbeg; h0 < hbeg + hlen; h0 += kRtH) {
    // activations: 64 rows x 8 chunks of 8 bf16, two chunks per thread
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int c = tid + 256 * i, row = c >> 3, seg = c & 7;
      const int t = t0 + row;
      uint4 v = make_uint4(0, 0, 0, 0);
      if (t < T) {
        v = *reinterpret_cast<const uint4*>(x + (size_t)t * H + h0 + seg * 8);
        if (x16 && blockIdx.y == 0) {
          const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
          uint32_t o[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const __half2 hh = __floats2half2_rn(__uint_as_float(w4[j] << 16), __uint_as_float(w4[j] & 0xffff0000u));
            o[j] = *reinterpret_cast<const uint32_t*>(&hh);
          }
          *reinterpret_cast<uint4*>(x16 + (size_t)t * H + h0 + seg * 8) = make_uint4(o[0], o[1], o[2], o[3]);
        }
      }
      *reinterpret_cast<uint4*>(xs + row * kRtPitch + seg * 8) = v;
    }
    // router: 64 rows x 16 float4, four per thread, each split into three bf16 parts
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int c = tid + 256 * i, row = c >> 4, seg = c & 15;
      const int e = e0 + row;
      float4 w = make_float4(0.f, 0.f, 0.f, 0.f);
      if (e < E) w = __ldg(reinterpret_cast<const float4*>(router + (size_t)e * H + h0 + seg * 4));
      const float wa[4] = {w.x, w.y, w.z, w.w};
      uint16_t p[3][4];
#pragma unroll
      for (int j = 0; j < 4; ++j) split3_bf16(wa[j], p[0][j], p[1][j], p[2][j]);
#pragma unroll
      for (int s = 0; s < 3; ++s)
        *reinterpret_cast<uint2*>(ws[s] + row * kRtPitch + seg * 4) =
            make_uint2(p[s][0] | (uint32_t)p[s][1] << 16, p[s][2] | (uint32_t)p[s][3] << 16);
    }
    __syncthreads();
#pragma unroll
    for (int ks = 0; ks < kRtH / 16; ++ks) {
      uint32_t a[4];
      ldmatrix_x4(a[0], a[1], a[2], a[3],
                  xs + (tg * 16 + ((lane >> 3) & 1) * 8 + (lane & 7)) * kRtPitch + ks * 16 + (lane >> 4) * 8);
#pragma unroll
      for (int s = 0; s < 3; ++s) {
#pragma unroll
        for (int j = 0; j < 4; j += 2) {  // column tiles j, j + 1
          uint32_t b0, b1, b2, b3;
          ldmatrix_x4(b0, b1, b2, b3,
                      ws[s] + (eh * 32 + (j + (lane >> 4)) * 8 + (lane & 7)) * kRtPitch + ks * 16 +
                          ((lane >> 3) & 1) * 8);
          mma_16816<true>(acc[j], a, b0, b1);
          mma_16816<true>(acc[j + 1], a, b2, b3);
        }
      }
    }
    __syncthreads();
  }
  const int g = lane >> 2, c2 = 2 * (lane & 3);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int t = t0 + tg * 16 + g + 8 * (i >> 1);
      const int e = e0 + eh * 32 + j * 8 + c2 + (i & 1);
      if (t < T && e < E) part[((size_t)hs * T + t) * E + e] = acc[j][i];
    }
  }
}

// ---- prefill-sized batches: split once, then a pipelined tensor-core GEMM ---------------
// At T >= kRtTiledMinT every token tile would re-split the whole router, so the split runs
// once per call into scratch (w3 = hi, mid, lo planes of bf16 [E, H]) and the logits GEMM
// streams x and w3 through a 4-stage cp.async ring of 32-h chunks.  Each thread accumulates
// the same exact products in the same fp32 order as in route_logits_kernel (16-h blocks in h
// order; hi, mid, lo within a block), so both kernels give identical logits.
constexpr int kRtH2 = 32;                                            // h per stage
constexpr int kRtPitch2 = 40;                                        // bf16 per staged row (32 + 8)
constexpr int kRtStages = 4;
constexpr int kRtStageBytes = (kRtTok + 3 * kRtExp) * kRtPitch2 * 2;  // x tile + three weight planes
constexpr int kRtSmem = kRtStages * kRtStageBytes;

// w3[s][e][h] (s = 0, 1, 2): the exact three-way bf16 split of router[e][h].
__global__ void route_split_kernel(const float* __restrict__ router, size_t n4, size_t plane,
                                   uint16_t* __restrict__ w3) {
  pdl_wait();
  pdl_trigger();
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x) {
    const float4 w = __ldg(reinterpret_cast<const float4*>(router) + i);
    const float wa[4] = {w.x, w.y, w.z, w.w};
    uint16_t p[3][4];
#pragma unroll
    for (int j = 0; j < 4; ++j) split3_bf16(wa[j], p[0][j], p[1][j], p[2][j]);
#pragma unroll
    for (int s = 0; s < 3; ++s)
      reinterpret_cast<uint2*>(w3 + s * plane)[i] =
          make_uint2(p[s][0] | (uint32_t)p[s][1] << 16, p[s][2] | (uint32_t)p[s][3] << 16);
  }
}

// part[hs][t][e] as route_logits_kernel, from the split planes.  Warp w owns tokens
// 16 (w & 3) .. + 15 and experts 32 (w >> 2) .. + 31 of the 64 x 64 CTA tile.
__global__ void __launch_bounds__(256) route_logits_tiled_kernel(const uint16_t* __restrict__ x,
                                                                 const uint16_t* __restrict__ w3, int T, int H, int E,
                                                                 int hsplit, float* __restrict__ part,
                                                                 int* __restrict__ counts,
                                                                 uint16_t* __restrict__ x16) {
  pdl_wait();
  pdl_trigger();
  extern __shared__ __align__(128) uint8_t rt_smem[];
  const int t0 = blockIdx.x * kRtTok, e0 = blockIdx.y * kRtExp, hs = blockIdx.z;
  const int hlen = H / hsplit, hbeg = hs * hlen, nsteps = hlen / kRtH2;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const size_t plane = (size_t)E * H;
  if (counts && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0)
    for (int e = tid; e < E; e += blockDim.x) counts[e] = 0;
  // one 16-byte chunk of the x tile and three of the weight planes per thread and stage
  const int lrow = tid >> 2, lseg = tid & 3;
  const int lt = t0 + lrow, le = e0 + lrow;
  const uint16_t* xsrc = x + (size_t)(lt < T ? lt : 0) * H + hbeg + lseg * 8;
  const uint16_t* wsrc = w3 + (size_t)(le < E ? le : 0) * H + hbeg + lseg * 8;
  auto load = [&](int step) {
    uint16_t* xs = reinterpret_cast<uint16_t*>(rt_smem + (step % kRtStages) * kRtStageBytes);
    const int h = step * kRtH2;
    cp_async16(xs + lrow * kRtPitch2 + lseg * 8, xsrc + h, lt < T);
#pragma unroll
    for (int s = 0; s < 3; ++s)
      cp_async16(xs + (kRtTok + s * kRtExp + lrow) * kRtPitch2 + lseg * 8, wsrc + s * plane + h, le < E);
  };
#pragma unroll
  for (int s = 0; s < kRtStages - 1; ++s) {
    if (s < nsteps) load(s);
    cp_async_commit();
  }
  const int tg = warp & 3, eh = warp >> 2;
  float acc[4][4];
#pragma unroll
  for (int j = 0; j < 4; ++j)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[j][i] = 0.f;
  for (int step = 0; step < nsteps; ++step) {
    cp_async_wait<kRtStages - 2>();
    __syncthreads();  // this stage landed for every thread; the stage refilled below is free
    if (step + kRtStages - 1 < nsteps) load(step + kRtStages - 1);
    cp_async_commit();
    const uint16_t* xs = reinterpret_cast<const uint16_t*>(rt_smem + (step % kRtStages) * kRtStageBytes);
    if (x16 && blockIdx.y == 0 && lt < T) {  // the f16 copy of this thread's chunk
      const uint4 v = *reinterpret_cast<const uint4*>(xs + lrow * kRtPitch2 + lseg * 8);
      const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
      uint32_t o[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const __half2 hh = __floats2half2_rn(__uint_as_float(w4[j] << 16), __uint_as_float(w4[j] & 0xffff0000u));
        o[j] = *reinterpret_cast<const uint32_t*>(&hh);
      }
      *reinterpret_cast<uint4*>(x16 + (size_t)lt * H + hbeg + step * kRtH2 + lseg * 8) =
          make_uint4(o[0], o[1], o[2], o[3]);
    }
#pragma unroll
    for (int ks = 0; ks < kRtH2 / 16; ++ks) {
      uint32_t a[4];
      ldmatrix_x4(a[0], a[1], a[2], a[3],
                  xs + (tg * 16 + ((lane >> 3) & 1) * 8 + (lane & 7)) * kRtPitch2 + ks * 16 + (lane >> 4) * 8);
#pragma unroll
      for (int s = 0; s < 3; ++s) {
        const uint16_t* ws = xs + (kRtTok + s * kRtExp) * kRtPitch2;
#pragma unroll
        for (int j = 0; j < 4; j += 2) {  // column tiles j, j + 1
          uint32_t b0, b1, b2, b3;
          ldmatrix_x4(b0, b1, b2, b3,
                      ws + (eh * 32 + (j + (lane >> 4)) * 8 + (lane & 7)) * kRtPitch2 + ks * 16 +
                          ((lane >> 3) & 1) * 8);
          mma_16816<true>(acc[j], a, b0, b1);
          mma_16816<true>(acc[j + 1], a, b2, b3);
        }
      }
    }
  }
  cp_async_wait<0>();
  const int g = lane >> 2, c2 = 2 * (lane & 3);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int t = t0 + tg * 16 + g + 8 * (i >> 1);
      const int e = e0 + eh * 32 + j * 8 + c2 + (i & 1);
      if (t < T && e < E) part[((size_t)hs * T + t) * E + e] = acc[j][i];
    }
  }
}

struct VI {
  float v;
  int i;
};

// Larger value wins; equal values -> lower index (the reference's strict '>' scan).
__device__ __forceinline__ bool better(float a, int ia, float b, int ib) { return a > b || (a == b && ia < ib); }

__device__ __forceinline__ VI warp_best(VI x) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, x.v, o);
    const int oi = __shfl_xor_sync(0xffffffffu, x.i, o);
    if (better(ov, oi, x.v, x.i)) {
      x.v = ov;
      x.i = oi;
    }
  }
  return x;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

constexpr int kMaxPerLane = 8;  // E <= 256
constexpr int kMaxTopK = 16;

// Selection and weights of one token from its logits v (lane + 32 i holds expert lane + 32 i,
// -inf beyond E), by one warp: the routing mode's selection score, top-k by repeated warp
// arg-max (ties to the lower index), the routing weights, and the writes of ids / weights /
// counts for token t.
template <int NPL>  // experts per lane: E <= 32 * NPL
__device__ __forceinline__ void select_topk(const float (&v)[NPL], int lane, int t, int E,
                                            const ccut_route_params& rp, int32_t* __restrict__ ids,
                                            float* __restrict__ weights, int* __restrict__ counts) {
  const int k = rp.top_k;
  // selection score
  float sel[NPL], sg[NPL];
  if (rp.mode == CCUT_ROUTE_SIGMOID_GROUP) {
    const int gsize = E / rp.n_group;
#pragma unroll
    for (int i = 0; i < NPL; ++i) {
      const int e = lane + 32 * i;
      sg[i] = e < E ? 1.f / (1.f + expf(-v[i])) : 0.f;
      sel[i] = e < E ? sg[i] + (rp.bias ? rp.bias[e] : 0.f) : -INFINITY;
    }
    // group score = sum of the two best selection scores in the group
    uint32_t keep = 0;
    float gscore_lane = -INFINITY;  // lane g holds the score of group g
    for (int g = 0; g < rp.n_group; ++g) {
      VI b1{-INFINITY, 0x7fffffff}, b2{-INFINITY, 0x7fffffff};
#pragma unroll
      for (int i = 0; i < NPL; ++i) {
        const int e = lane + 32 * i;
        if (e < E && e / gsize == g) {
          if (better(sel[i], e, b1.v, b1.i)) {
            b2 = b1;
            b1 = VI{sel[i], e};
          } else if (better(sel[i], e, b2.v, b2.i)) {
            b2 = VI{sel[i], e};
          }
        }
      }
      // merge top-2 across the warp
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        VI c1{__shfl_xor_sync(0xffffffffu, b1.v, o), __shfl_xor_sync(0xffffffffu, b1.i, o)};
        VI c2{__shfl_xor_sync(0xffffffffu, b2.v, o), __shfl_xor_sync(0xffffffffu, b2.i, o)};
        VI n1, n2;
        if (better(c1.v, c1.i, b1.v, b1.i)) {
          n1 = c1;
          n2 = better(b1.v, b1.i, c2.v, c2.i) ? b1 : c2;
        } else {
          n1 = b1;
          n2 = better(c1.v, c1.i, b2.v, b2.i) ? c1 : b2;
        }
        b1 = n1;
        b2 = n2;
      }
      if (lane == g) gscore_lane = b1.v + b2.v;
    }
    for (int r = 0; r < rp.topk_group; ++r) {
      VI b = warp_best(VI{lane < rp.n_group && !((keep >> lane) & 1) ? gscore_lane : -INFINITY,
                          lane < rp.n_group ? lane : 0x7fffffff});
      keep |= 1u << b.i;
    }
#pragma unroll
    for (int i = 0; i < NPL; ++i) {
      const int e = lane + 32 * i;
      if (e < E && !((keep >> (e / gsize)) & 1)) sel[i] = -INFINITY;
    }
  } else {
#pragma unroll
    for (int i = 0; i < NPL; ++i) {
      sel[i] = v[i];
      sg[i] = 0.f;
    }
  }
  // top-k by repeated warp arg-max
  uint32_t used = 0;
  int my_id = -1;
  float my_logit = 0.f, my_sig = 0.f;  // lane j < k keeps pick j
  for (int j = 0; j < k; ++j) {
    VI b{-INFINITY, 0x7fffffff};
#pragma unroll
    for (int i = 0; i < NPL; ++i) {
      const int e = lane + 32 * i;
      if (e < E && !((used >> i) & 1) && better(sel[i], e, b.v, b.i)) b = VI{sel[i], e};
    }
    b = warp_best(b);
    float lg = 0.f, sgv = 0.f;
#pragma unroll
    for (int i = 0; i < NPL; ++i) {
      if (lane + 32 * i == b.i) {
        used |= 1u << i;
        lg = v[i];
        sgv = sg[i];
      }
    }
    const int owner = b.i & 31;
    lg = __shfl_sync(0xffffffffu, lg, owner);
    sgv = __shfl_sync(0xffffffffu, sgv, owner);
    if (lane == j) {
      my_id = b.i;
      my_logit = lg;
      my_sig = sgv;
    }
  }
  float w = 0.f;
  if (rp.mode == CCUT_ROUTE_SOFTMAX_TOPK) {
    // softmax over all E, keep the k picks (no renormalisation)
    const float m = __shfl_sync(0xffffffffu, my_logit, 0);  // pick 0 is the max logit
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < NPL; ++i)
      if (lane + 32 * i < E) s += expf(v[i] - m);
    s = warp_sum(s);
    w = expf(my_logit - m) / fmaxf(s, 1e-30f);
  } else if (rp.mode == CCUT_ROUTE_TOPK_SOFTMAX) {
    const float m = __shfl_sync(0xffffffffu, my_logit, 0);
    const float ex = lane < k ? expf(my_logit - m) : 0.f;
    const float s = warp_sum(ex);
    w = ex / fmaxf(s, 1e-30f);
  } else {
    const float s = warp_sum(lane < k ? my_sig : 0.f);
    w = my_sig / (s + 1e-20f) * rp.routed_scaling;
  }
  if (my_id < 0 || my_id >= E) {  // no finite score left (NaN logits): route nowhere
    my_id = 0;
    w = 0.f;
  }
  if (lane < k) {
    ids[(size_t)t * k + lane] = my_id;
    weights[(size_t)t * k + lane] = w;
    if (counts) atomicAdd(&counts[my_id], 1);
  }}

// One warp per token.  Logits come either from `part` (hsplit partial sums) or `logits_in`.
template <int NPL>
__global__ void __launch_bounds__(256) route_topk_kernel(const float* __restrict__ part, int hsplit,
                                                         const float* __restrict__ logits_in, int T, int E,
                                                         ccut_route_params rp, int32_t* __restrict__ ids,
                                                         float* __restrict__ weights, float* __restrict__ logits_out,
                                                         int* __restrict__ counts) {
  pdl_wait();
  pdl_trigger();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x * 8 + warp;
  if (t >= T) return;
  float v[NPL];
#pragma unroll
  for (int i = 0; i < NPL; ++i) {
    const int e = lane + 32 * i;
    float val = -INFINITY;
    if (e < E) {
      if (logits_in) {
        val = logits_in[(size_t)t * E + e];
      } else {
        // eight independent partial sums keep eight loads in flight per lane
        const float* pp = part + (size_t)t * E + e;
        const size_t ps = (size_t)T * E;
        float a8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        int s = 0;
        for (; s + 8 <= hsplit; s += 8) {
#pragma unroll
          for (int j = 0; j < 8; ++j) a8[j] += pp[(size_t)(s + j) * ps];
        }
        for (; s < hsplit; ++s) a8[0] += pp[(size_t)s * ps];
        val = ((a8[0] + a8[1]) + (a8[2] + a8[3])) + ((a8[4] + a8[5]) + (a8[6] + a8[7]));
      }
      if (logits_out) logits_out[(size_t)t * E + e] = val;
    }
    v[i] = val;
  }
  select_topk(v, lane, t, E, rp, ids, weights, counts);
}

// Decode-sized calls (T <= kTopkWideMaxT) with partial sums: one CTA per token, so that the
// H-split partial sums are read by 256 threads of T CTAs rather than one warp per token.
// Thread (j, e) sums the splits s = j, j + 8, ... of expert e (split j = 0 also takes the
// hsplit % 8 tail), and the eight sums are added in the same tree as route_topk_kernel, so
// the logits (and hence the routing) are bit-identical to it.
constexpr int kTopkWideMaxT = 256;

template <int NPL>
__global__ void __launch_bounds__(256) route_topk_wide_kernel(const float* __restrict__ part, int hsplit, int T,
                                                              int E, ccut_route_params rp, int32_t* __restrict__ ids,
                                                              float* __restrict__ weights,
                                                              float* __restrict__ logits_out,
                                                              int* __restrict__ counts) {
  pdl_wait();
  pdl_trigger();
  __shared__ float a8s[8][kMaxPerLane * 32];
  __shared__ float lg[kMaxPerLane * 32];
  const int t = blockIdx.x, tid = threadIdx.x;
  const size_t ps = (size_t)T * E;
  const int main = hsplit / 8 * 8;
  for (int idx = tid; idx < 8 * E; idx += blockDim.x) {
    const int j = idx / E, e = idx - j * E;
    const float* pp = part + (size_t)t * E + e;
    float a = 0.f;
    for (int s = j; s < main; s += 8) a += pp[(size_t)s * ps];
    if (j == 0)
      for (int s = main; s < hsplit; ++s) a += pp[(size_t)s * ps];
    a8s[j][e] = a;
  }
  __syncthreads();
  for (int e = tid; e < E; e += blockDim.x) {
    const float val = ((a8s[0][e] + a8s[1][e]) + (a8s[2][e] + a8s[3][e])) +
                      ((a8s[4][e] + a8s[5][e]) + (a8s[6][e] + a8s[7][e]));
    lg[e] = val;
    if (logits_out) logits_out[(size_t)t * E + e] = val;
  }
  __syncthreads();
  if (tid >= 32) return;
  float v[NPL];
#pragma unroll
  for (int i = 0; i < NPL; ++i) {
    const int e = tid + 32 * i;
    v[i] = e < E ? lg[e] : -INFINITY;
  }
  select_topk(v, tid, t, E, rp, ids, weights, counts);
}

// Stable counting sort of the T*k (token, slot) pairs by expert, one CTA per contiguous
// chunk of pairs.  A pair's row is offsets[e] + (pairs of expert e before its chunk) +
// (pairs of expert e before it inside the chunk).  The first term is an exclusive scan of
// `counts`; the second a shared-memory histogram of the pairs before the chunk (or, for the
// later half of the chunks, `counts` minus the histogram of the pairs from the chunk on);
// the third comes from rounds of 256 pairs: __match_any_sync ranks a pair inside its warp
// and per-warp counters in shared memory rank the warps.  Pair ids outside [0, E) take no
// row (their pair_row is -1), so the V valid pairs fill rows [0, V) and the shared-expert
// slices follow at V + s * T (V = T * k when every id is valid).
constexpr int kPermThreads = 256;
constexpr int kPermWarps = kPermThreads / 32;

__global__ void __launch_bounds__(kPermThreads) permute_kernel(
    const int32_t* __restrict__ ids, const float* __restrict__ weights, int T, int k, int E, int slices,
    float shared_gate, const int* __restrict__ counts, int chunk, int32_t* __restrict__ offsets,
    int32_t* __restrict__ row_token, float* __restrict__ row_weight, int32_t* __restrict__ pair_row) {
  pdl_wait();
  pdl_trigger();
  __shared__ int base[kMaxExperts];
  __shared__ int hist[kMaxExperts];
  __shared__ int wcnt[kPermWarps][kMaxExperts];
  __shared__ int s_valid;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int tk = T * k;
  const int c0 = min(tk, blockIdx.x * chunk), c1 = min(tk, c0 + chunk);
  for (int e = tid; e < E; e += kPermThreads) {
    hist[e] = 0;
#pragma unroll
    for (int w = 0; w < kPermWarps; ++w) wcnt[w][e] = 0;
  }
  if (warp == 0) {  // exclusive scan of counts -> base (= offsets)
    int carry = 0;
    for (int b = 0; b < E; b += 32) {
      const int e = b + lane;
      const int c = e < E ? counts[e] : 0;
      int inc = c;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int u = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += u;
      }
      if (e < E) base[e] = carry + inc - c;
      carry += __shfl_sync(0xffffffffu, inc, 31);
    }
    if (lane == 0) s_valid = carry;
  }
  __syncthreads();
  const int valid = s_valid;
  if (blockIdx.x == 0) {
    for (int e = tid; e < E; e += kPermThreads) offsets[e] = base[e];
    for (int s = tid; s <= slices; s += kPermThreads) offsets[E + s] = valid + s * T;
  }
  // pairs of each expert before the chunk
  const bool from_front = c0 <= tk - c0;
  const int h0 = from_front ? 0 : c0, h1 = from_front ? c0 : tk;
  for (int i = h0 + tid; i < h1; i += kPermThreads) {
    const int e = ids[i];
    if (e >= 0 && e < E) atomicAdd(&hist[e], 1);
  }
  __syncthreads();
  for (int e = tid; e < E; e += kPermThreads) base[e] += from_front ? hist[e] : counts[e] - hist[e];
  __syncthreads();
  const unsigned lt = (1u << lane) - 1u;
  for (int r0 = c0; r0 < c1; r0 += kPermThreads) {
    const int i = r0 + tid;
    int e = i < c1 ? ids[i] : -1;
    if (e >= E) e = -1;
    const float wt = e >= 0 ? weights[i] : 0.f;
    const unsigned same = __match_any_sync(0xffffffffu, e);
    if (e >= 0 && (same & lt) == 0) wcnt[warp][e] = __popc(same);
    __syncthreads();
    if (e >= 0) {
      int p = base[e] + __popc(same & lt);
      for (int w = 0; w < warp; ++w) p += wcnt[w][e];
      row_token[p] = i / k;
      row_weight[p] = wt;
      pair_row[i] = p;
    } else if (i < c1) {
      pair_row[i] = -1;
    }
    __syncthreads();
    for (int ee = tid; ee < E; ee += kPermThreads) {
      int add = 0;
#pragma unroll
      for (int w = 0; w < kPermWarps; ++w) {
        add += wcnt[w][ee];
        wcnt[w][ee] = 0;
      }
      base[ee] += add;
    }
    __syncthreads();
  }
  // shared-expert rows: every token once per slice
  const int nsh = slices * T;
  for (int r = blockIdx.x * kPermThreads + tid; r < nsh; r += gridDim.x * kPermThreads) {
    row_token[valid + r] = r % T;
    row_weight[valid + r] = shared_gate;
  }
}

int launch_route(const uint16_t* x, const float* router, int T, int H, int E, const ccut_route_params& rp,
                 int32_t* ids, float* weights, float* logits, float* part, int* counts, uint16_t* x16,
                 cudaStream_t st) {
  const int hs = route_hsplit(T, E, H);
  dim3 g1((T + kRtTok - 1) / kRtTok, (E + kRtExp - 1) / kRtExp, hs);
  int rc;
  if (T >= kRtTiledMinT) {  // the split planes follow the partial sums in `part`
    uint16_t* w3 = reinterpret_cast<uint16_t*>(part + ((size_t)hs * T * E + 3) / 4 * 4);
    const size_t n4 = (size_t)E * H / 4;
    size_t blocks = (n4 + 255) / 256;
    if (blocks > 148 * 8) blocks = 148 * 8;
    rc = launch_k(route_split_kernel, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, st, router, n4,
                  (size_t)E * H, w3);
    if (rc) return rc;
    static std::atomic<uint64_t> smem_set{0};
    rc = ensure_smem_limit(route_logits_tiled_kernel, kRtSmem, smem_set);
    if (rc) return rc;
    rc = launch_k(route_logits_tiled_kernel, g1, dim3(256), kRtSmem, st, x, (const uint16_t*)w3, T, H, E, hs, part,
                  counts, x16);
  } else {
    rc = launch_k(route_logits_kernel, g1, dim3(256), 0, st, x, router, T, H, E, hs, part, counts, x16);
  }
  if (rc) return rc;
  const bool narrow = E <= 128;  // four experts per lane instead of eight
  if (T <= kTopkWideMaxT)
    return launch_k(narrow ? route_topk_wide_kernel<4> : route_topk_wide_kernel<kMaxPerLane>, dim3(T), dim3(256), 0,
                    st, (const float*)part, hs, T, E, rp, ids, weights, logits, counts);
  return launch_k(narrow ? route_topk_kernel<4> : route_topk_kernel<kMaxPerLane>, dim3((T + 7) / 8), dim3(256), 0, st,
                  (const float*)part, hs, (const float*)nullptr, T, E, rp, ids, weights, logits, counts);
}

int launch_topk(const float* logits, int T, int E, const ccut_route_params& rp, int32_t* ids, float* weights,
                cudaStream_t st) {
  return launch_k(E <= 128 ? route_topk_kernel<4> : route_topk_kernel<kMaxPerLane>, dim3((T + 7) / 8), dim3(256), 0,
                  st, (const float*)nullptr, 0, logits, T, E, rp, ids, weights, (float*)nullptr, (int*)nullptr);
}

int launch_permute(const int32_t* ids, const float* weights, int T, int k, int E, int slices, float shared_gate,
                   const int* counts, int32_t* offsets, int32_t* row_token, float* row_weight, int32_t* pair_row,
                   cudaStream_t st) {
  // about one wave of CTAs; chunks are whole rounds of kPermThreads pairs
  const int tk = T * k;
  const int per = (tk + 147) / 148;
  const int chunk = (per + kPermThreads - 1) / kPermThreads * kPermThreads;
  int blocks = chunk > 0 ? (tk + chunk - 1) / chunk : 1;
  if (blocks < 1) blocks = 1;
  return launch_k(permute_kernel, dim3(blocks), dim3(kPermThreads), 0, st, ids, weights, T, k, E, slices, shared_gate,
                  counts, chunk > 0 ? chunk : kPermThreads, offsets, row_token, row_weight, pair_row);
}

// counts[e] from ids (used when the caller supplies its own routing).
__global__ void count_kernel(const int32_t* __restrict__ ids, int n, int E, int* __restrict__ counts) {
  pdl_wait();
  pdl_trigger();
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const int e = ids[i];
    if (e >= 0 && e < E) atomicAdd(&counts[e], 1);
  }
}

int launch_count(const int32_t* ids, int n, int E, int* counts, cudaStream_t st) {
  if (cudaMemsetAsync(counts, 0, sizeof(int) * E, st) != cudaSuccess) return CCUT_ERR_CUDA;
  int blocks = (n + 255) / 256;
  if (blocks > 1024) blocks = 1024;
  if (blocks < 1) blocks = 1;
  return launch_k(count_kernel, dim3(blocks), dim3(256), 0, st, ids, n, E, counts);
}

}  // namespace ccut
