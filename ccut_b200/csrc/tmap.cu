// tmap.cu -- TMA tensor maps for the activation operand, and the row gather that feeds it.
//
// The activation rows of the grouped GEMM must be contiguous per expert for tiled TMA
// loads, so the gate/up input is first gathered into expert-sorted order: xp[r] =
// x[row_token[r]], bf16 as given (the MMA operand type).
#include <cudaTypedefs.h>

#include "kernels.cuh"

namespace ccut {

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

int encode_rows_map(CUtensorMap* map, const void* base, int rows, int cols, int box_rows) {
  auto fn = encode_fn();
  if (!fn) return CCUT_ERR_CUDA;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (cols * 2) % 16 || rows < 1) return CCUT_ERR_INVALID;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)cols * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? CCUT_OK : CCUT_ERR_CUDA;
}

__global__ void gather_rows_kernel(const uint16_t* __restrict__ x, const int32_t* __restrict__ row_token, int R,
                                   const int* __restrict__ nrows, int H, uint16_t* __restrict__ xp) {
  pdl_wait();
  pdl_trigger();
  const int per_row = H / 8;
  if (nrows && *nrows < R) R = *nrows;  // rows the permutation actually produced
  const size_t total = (size_t)R * per_row;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int r = static_cast<int>(i / per_row), c = static_cast<int>(i % per_row);
    const int t = row_token ? row_token[r] : r;
    *reinterpret_cast<uint4*>(xp + (size_t)r * H + 8 * c) = *reinterpret_cast<const uint4*>(x + (size_t)t * H + 8 * c);
  }
}

int launch_gather_rows(const uint16_t* x_bf16, const int32_t* row_token, int R, const int* nrows, int H,
                       uint16_t* xp, cudaStream_t st) {
  size_t total = (size_t)R * (H / 8);
  size_t blocks = (total + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  if (blocks < 1) blocks = 1;
  return launch_k(gather_rows_kernel, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, st, x_bf16, row_token, R,
                  nrows, H, xp);
}

}  // namespace ccut
