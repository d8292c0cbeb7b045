// host.cuh -- host-side helpers shared by the C-ABI translation units (capi.cu, ep.cu):
// argument checks, workspace carving and the expert-FFN driver.
#pragma once

#include "kernels.cuh"

namespace ccut {

constexpr int kMaxTopK = 16;
constexpr int kMaxRoutedExperts = 256;

// Carves 256-byte aligned regions out of a caller workspace (base == nullptr: sizing pass).
struct Carver {
  uint8_t* base;
  size_t off = 0;
  explicit Carver(void* b) : base(static_cast<uint8_t*>(b)) {}
  template <class T>
  T* take(size_t n) {
    off = (off + 255) / 256 * 256;
    T* p = base ? reinterpret_cast<T*>(base + off) : nullptr;
    off += n * sizeof(T);
    return p;
  }
};

// Expert-FFN scratch.  Row layout (tcgen05): xp = bf16 activations gathered in expert
// order [R, H].  Fragment layout (mma.sync): x16 = f16 copy of x [T, H].
// Both: intermediate rows [R, I] (bf16 from tcgen05, f16 from mma.sync).
struct FfnScratch {
  uint16_t* x16;
  uint16_t* xp;
  uint16_t* hbuf;
  int* sched;  // work counters of the mma.sync GEMM (null: static schedule)
};

// Work counters of the mma.sync grouped GEMM's dynamic schedule (gemm.cu).  Every workspace
// that runs that GEMM keeps them right after its status word, at an offset that does not
// depend on the call's shapes, so that a workspace reused for other shapes still finds them
// zero: the caller zero-fills a workspace before its first use and every launch leaves the
// counters zero.
constexpr int kSchedInts = 64;
inline int* take_sched(Carver& c) { return c.take<int>(kSchedInts); }

int num_sms();
bool valid_fmt(int f);
int check_layer(const ccut_moe_layer* L);
int check_route(const ccut_route_params* rp, int E);
// Mean rows per routed expert of a call (T tokens, top-k over the layer's experts).
long mean_rows(const ccut_moe_layer* L, int T, int k);
// Kernel policy: tcgen05 (true) or mma.sync (false) for a mean of per_expert rows.
bool use_tc(const ccut_moe_layer* L, long per_expert);
size_t rows_of(const ccut_moe_layer* L, int T, int k);
// sched: this FFN's GEMM work counters (take_sched), or null for the static schedule.
FfnScratch carve_ffn(Carver& c, const ccut_moe_layer* L, int T, int k, bool with_input, int* sched);
// gate/up then down over the rows of a permutation; x16 must already hold x in f16 when
// the mma.sync kernel runs.  y_rows: the weighted rows, fp32 or (y_bf16) bf16.
int run_ffn(const ccut_moe_layer* L, long per_expert, const uint16_t* x, const FfnScratch& s, int T, int k,
            const int32_t* offsets, const int32_t* row_token, const float* row_weight, void* y_rows, int y_bf16,
            int* status, cudaStream_t st);

}  // namespace ccut
