// combine.cu -- weighted un-permute: out[t] = sum_j y[pair_row[t, j]] + sum_s y[shared row].
//
// The rows already carry their routing weight (applied in the down-projection epilogue),
// so this is a fixed-order fp32 sum per token: deterministic, no atomics.  The rows are
// fp32, or bf16 when the fused forward produces a bf16 output (one rounding of each
// weighted row, half the bytes written by the down GEMM and read here).  Follows the
// scatter-add of ccut/models/generic.py:377-378 and the shared-expert add of
// ccut/models/generic.py:380-385.
#include "launch.cuh"
#include "layout.cuh"

namespace ccut {

constexpr int kCombThreads = 256;
constexpr int kCombMaxRows = 16 + CCUT_MAX_SHARED_SLICES;  // top-k + shared slices

// One CTA per (token, 1024-column chunk).  The token's source rows are staged in shared
// memory first, so every lane's row loads are independent of one another; the sum runs in
// the fixed order j = 0..k-1, then the shared slices.
template <bool kBf16In, bool kBf16Out>
__global__ void __launch_bounds__(kCombThreads) combine_kernel(const void* __restrict__ y,
                                                               const int32_t* __restrict__ pair_row, int T, int k,
                                                               int H, int slices, int shared_base,
                                                               void* __restrict__ out) {
  pdl_wait();
  pdl_trigger();
  __shared__ int rows[kCombMaxRows];
  const int t = blockIdx.x;
  const int R = shared_base + slices * T;
  if (threadIdx.x < k) {
    const int p = pair_row[(size_t)t * k + threadIdx.x];
    rows[threadIdx.x] = (p >= 0 && p < R) ? p : -1;
  } else if (threadIdx.x < k + slices) {
    rows[threadIdx.x] = shared_base + (threadIdx.x - k) * T + t;
  }
  __syncthreads();
  const int n = k + slices;
  const int h4n = H / 4;
  const int h4 = blockIdx.y * kCombThreads + threadIdx.x;
  if (h4 >= h4n) return;
  float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 4
  for (int j = 0; j < n; ++j) {
    const int p = rows[j];
    if (p >= 0) {
      float4 v;
      if constexpr (kBf16In) {  // 4 bf16 -> fp32 (exact)
        const uint2 u = reinterpret_cast<const uint2*>(y)[(size_t)p * h4n + h4];
        v = make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xffff0000u), __uint_as_float(u.y << 16),
                        __uint_as_float(u.y & 0xffff0000u));
      } else {
        v = reinterpret_cast<const float4*>(y)[(size_t)p * h4n + h4];
      }
      s.x += v.x;
      s.y += v.y;
      s.z += v.z;
      s.w += v.w;
    }
  }
  if constexpr (kBf16Out) {
    __nv_bfloat162 a = __floats2bfloat162_rn(s.x, s.y);
    __nv_bfloat162 b = __floats2bfloat162_rn(s.z, s.w);
    uint2 pk;
    pk.x = *reinterpret_cast<uint32_t*>(&a);
    pk.y = *reinterpret_cast<uint32_t*>(&b);
    reinterpret_cast<uint2*>(static_cast<uint16_t*>(out) + (size_t)t * H)[h4] = pk;
  } else {
    reinterpret_cast<float4*>(static_cast<float*>(out) + (size_t)t * H)[h4] = s;
  }
}

// y: the weighted rows, fp32 or (y_bf16) bf16.
int launch_combine(const void* y, int y_bf16, const int32_t* pair_row, int T, int k, int H, int slices, int shared_base,
                   void* out, int out_dtype, cudaStream_t st) {
  if (k < 1 || slices < 0 || k + slices > kCombMaxRows || H % 4) return CCUT_ERR_UNSUPPORTED;
  if (T == 0) return CCUT_OK;
  if (shared_base < 0) shared_base = T * k;
  const dim3 grid(T, (H / 4 + kCombThreads - 1) / kCombThreads);
  const bool bo = out_dtype == CCUT_OUT_BF16;
  auto kern = y_bf16 ? (bo ? combine_kernel<true, true> : combine_kernel<true, false>)
                     : (bo ? combine_kernel<false, true> : combine_kernel<false, false>);
  return launch_k(kern, grid, dim3(kCombThreads), 0, st, y, pair_row, T, k, H, slices, shared_base, out);
}

// bf16 -> f16 copy (FP8 path operands are f16).
__global__ void bf16_to_f16_kernel(const uint16_t* __restrict__ in, uint16_t* __restrict__ out, size_t n) {
  pdl_wait();
  pdl_trigger();
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const float v = __uint_as_float(static_cast<uint32_t>(in[i]) << 16);
    out[i] = __half_as_ushort(__float2half_rn(v));
  }
}

int launch_bf16_to_f16(const uint16_t* in, uint16_t* out, size_t n, cudaStream_t st) {
  size_t blocks = (n + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  if (blocks < 1) blocks = 1;
  return launch_k(bf16_to_f16_kernel, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, st, in, out, n);
}

__global__ void fill_offsets_kernel(int32_t* off, int m) {
  pdl_wait();
  pdl_trigger();
  off[0] = 0;
  off[1] = m;
}

int launch_fill_offsets(int32_t* off, int m, cudaStream_t st) {
  return launch_k(fill_offsets_kernel, dim3(1), dim3(1), 0, st, off, m);
}

}  // namespace ccut
