// combine.cu -- weighted un-permute: out[t] = sum_j y[pair_row[t, j]] + sum_s y[shared row].
//
// The rows already carry their routing weight (applied in the down-projection epilogue),
// so this is a fixed-order fp32 sum per token: deterministic, no atomics.  Follows the
// scatter-add of ccut/models/generic.py:377-378 and the shared-expert add of
// ccut/models/generic.py:380-385.
#include "layout.cuh"

namespace ccut {

template <bool kBf16Out>
__global__ void __launch_bounds__(256) combine_kernel(const float* __restrict__ y, const int32_t* __restrict__ pair_row,
                                                      int T, int k, int H, int slices, void* __restrict__ out) {
  const int t = blockIdx.x;
  const int tk = T * k;
  const int R = tk + slices * T;
  const int h4n = H / 4;
  for (int h4 = threadIdx.x; h4 < h4n; h4 += blockDim.x) {
    float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int j = 0; j < k; ++j) {
      const int p = pair_row[(size_t)t * k + j];
      if (p >= 0 && p < R) {
        const float4 v = reinterpret_cast<const float4*>(y + (size_t)p * H)[h4];
        s.x += v.x;
        s.y += v.y;
        s.z += v.z;
        s.w += v.w;
      }
    }
    for (int sl = 0; sl < slices; ++sl) {
      const float4 v = reinterpret_cast<const float4*>(y + (size_t)(tk + sl * T + t) * H)[h4];
      s.x += v.x;
      s.y += v.y;
      s.z += v.z;
      s.w += v.w;
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
}

int launch_combine(const float* y, const int32_t* pair_row, int T, int k, int H, int slices, void* out,
                   int out_dtype, cudaStream_t st) {
  if (out_dtype == CCUT_OUT_BF16)
    combine_kernel<true><<<T, 256, 0, st>>>(y, pair_row, T, k, H, slices, out);
  else
    combine_kernel<false><<<T, 256, 0, st>>>(y, pair_row, T, k, H, slices, out);
  return cudaPeekAtLastError() == cudaSuccess ? CCUT_OK : CCUT_ERR_CUDA;
}

// bf16 -> f16 copy (FP8 path operands are f16).
__global__ void bf16_to_f16_kernel(const uint16_t* __restrict__ in, uint16_t* __restrict__ out, size_t n) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const float v = __uint_as_float(static_cast<uint32_t>(in[i]) << 16);
    out[i] = __half_as_ushort(__float2half_rn(v));
  }
}

int launch_bf16_to_f16(const uint16_t* in, uint16_t* out, size_t n, cudaStream_t st) {
  size_t blocks = (n + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  if (blocks < 1) blocks = 1;
  bf16_to_f16_kernel<<<static_cast<int>(blocks), 256, 0, st>>>(in, out, n);
  return cudaPeekAtLastError() == cudaSuccess ? CCUT_OK : CCUT_ERR_CUDA;
}

__global__ void fill_offsets_kernel(int32_t* off, int m) {
  off[0] = 0;
  off[1] = m;
}

int launch_fill_offsets(int32_t* off, int m, cudaStream_t st) {
  fill_offsets_kernel<<<1, 1, 0, st>>>(off, m);
  return cudaPeekAtLastError() == cudaSuccess ? CCUT_OK : CCUT_ERR_CUDA;
}

}  // namespace ccut
