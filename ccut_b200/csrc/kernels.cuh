// kernels.cuh -- host-side launchers implemented in the .cu files, used by capi.cu.
#pragma once

#include "launch.cuh"
#include "layout.cuh"

namespace ccut {

enum { kFfn1 = 0, kFfn2 = 1 };

struct GemmArgs {
  const uint8_t* w;      // packed weights of expert 0
  size_t expert_stride;  // bytes between experts
  int K, N;              // inputs, outputs of one matrix
  const uint16_t* x;     // activation rows (bf16 for AWQ, f16 for FP8)
  int x_ld;              // elements per activation row
  const int* row_src;    // activation row of each GEMM row, or null (identity)
  const int* offsets;    // [num_e + 1] first GEMM row of each expert
  int num_e;
  void* out;
  int out_ld;
  const float* row_weight;  // FFN2: per-row multiplier (null -> 1)
  int* status;
  // Dynamic scheduling (gemm.cu): sched[0] hands out work items, sched[1] counts the CTAs
  // done; both zero on entry, left zero on exit.  Null: static item striding.
  int* sched;
  int out_bf16 = 0;  // FFN2: weighted rows as bf16 (one rounding) instead of fp32
};

// Arguments of the tcgen05 grouped GEMM (tc_gemm.cu); the activation operand arrives
// through a TMA tensor map passed separately.
struct TcArgs {
  const uint8_t* w;      // packed weights (row layout) of expert 0
  size_t expert_stride;  // bytes between experts
  int K, N;              // inputs, outputs of one matrix
  const int* offsets;    // [num_e + 1] first GEMM row of each expert
  int num_e;
  void* out;
  int out_ld;
  const float* row_weight;
  int* status;
  int out_bf16 = 0;  // FFN2: weighted rows as bf16 (one rounding) instead of fp32
  // Dynamic item schedule: sched[0] hands out work items, sched[1] counts the clusters done;
  // both zero on entry, left zero on exit (the same counters as GemmArgs::sched).  Null:
  // static item striding.
  int* sched = nullptr;
};

// tc_gemm.cu: the activation operand `map` covers bf16 rows [R, K] in expert order (boxes
// of 64 x 128, encode_rows_map)
int launch_tc_gemm(int fmt, int mode, const CUtensorMap& map, const TcArgs& a, int num_sms, cudaStream_t st);
// tmap.cu: 2-D bf16 tensor map over a row-major [rows, cols] buffer, boxes of 64 x box_rows,
// 128-byte swizzle (host side)
int encode_rows_map(CUtensorMap* map, const void* base, int rows, int cols, int box_rows);
constexpr int kTcBoxRows = 128;  // token rows per CTA and stage of the tcgen05 GEMM
// xp[r] = x[row_token[r]] (bf16 rows in expert order); nrows: device row count bound (rows
// >= *nrows are left alone), or null
int launch_gather_rows(const uint16_t* x_bf16, const int32_t* row_token, int R, const int* nrows, int H,
                       uint16_t* xp, cudaStream_t st);

// pack.cu
int launch_pack(int fmt, int layout, const void* q, const void* z, const void* s, int K, int N, int nibble_order,
                void* dst, int nmat, int slot, cudaStream_t st);
int launch_dequant(int fmt, int layout, const void* packed, int K, int N, int nmat, int slot, float* out,
                   cudaStream_t st);
// route.cu
int route_hsplit(int T, int E, int H);
size_t route_scratch_floats(int T, int E, int H);  // the `part` scratch launch_route needs
size_t route_scratch_floats_upto(int T_cap, int E, int H);  // enough for every T <= T_cap
int launch_route(const uint16_t* x, const float* router, int T, int H, int E, const ccut_route_params& rp,
                 int32_t* ids, float* weights, float* logits, float* part, int* counts, uint16_t* x16,
                 cudaStream_t st);
int launch_topk(const float* logits, int T, int E, const ccut_route_params& rp, int32_t* ids, float* weights,
                cudaStream_t st);
int launch_permute(const int32_t* ids, const float* weights, int T, int k, int E, int slices, float shared_gate,
                   const int* counts, int32_t* offsets, int32_t* row_token, float* row_weight, int32_t* pair_row,
                   cudaStream_t st);
int launch_count(const int32_t* ids, int n, int E, int* counts, cudaStream_t st);
// gemm.cu
int launch_gemm(int fmt, int mode, int mt, const GemmArgs& a, int num_sms, cudaStream_t st);
// combine.cu
// shared rows of slice s sit at shared_base + s * T (shared_base < 0: T * k)
int launch_combine(const void* y, int y_bf16, const int32_t* pair_row, int T, int k, int H, int slices, int shared_base,
                   void* out, int out_dtype, cudaStream_t st);
int launch_bf16_to_f16(const uint16_t* in, uint16_t* out, size_t n, cudaStream_t st);
int launch_fill_offsets(int32_t* off, int m, cudaStream_t st);

}  // namespace ccut
