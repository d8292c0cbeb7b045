// capi.cu -- extern "C" entry points of libccut_moe.so (declared in include/ccut_moe.h).
//
// Argument checks happen here, on the host, before anything is enqueued; kernels never
// see a shape they were not written for.  Workspaces are carved into 256-byte aligned
// regions; the first region is the device status word of ccut_workspace_status().
#include <cstdlib>

#include "host.cuh"

namespace ccut {

int num_sms() {
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (!cache[dev]) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    cache[dev] = n > 0 ? n : 148;
  }
  return cache[dev];
}

thread_local bool g_pdl_on = false;

bool pdl_enabled() {
  static const bool on = [] {
    const char* v = getenv("CCUT_PDL");
    return !(v && v[0] == '0');
  }();
  return on;
}

bool valid_fmt(int f) {
  return f == CCUT_FMT_AWQ_INT4_G128 || f == CCUT_FMT_FP8_E4M3_B128 || f == CCUT_FMT_FP8_E4M3_CH ||
         f == CCUT_FMT_INT4_SYM_G128;
}

int check_layer(const ccut_moe_layer* L) {
  if (!L) return CCUT_ERR_INVALID;
  if (!valid_fmt(L->format)) return CCUT_ERR_UNSUPPORTED;
  if (L->kernel != CCUT_KERNEL_AUTO && L->kernel != CCUT_KERNEL_TC && L->kernel != CCUT_KERNEL_MMA)
    return CCUT_ERR_UNSUPPORTED;
  if (L->kernel == CCUT_KERNEL_MMA && (!L->w13_frags || !L->w2_frags)) return CCUT_ERR_INVALID;
  if (L->hidden <= 0 || L->inter <= 0 || L->hidden % 128 || L->inter % 128) return CCUT_ERR_INVALID;
  if (L->num_experts < 1 || L->num_experts > kMaxRoutedExperts) return CCUT_ERR_UNSUPPORTED;
  if (L->num_shared_slices < 0 || L->num_shared_slices > CCUT_MAX_SHARED_SLICES ||
      L->num_experts + L->num_shared_slices > kMaxExperts)
    return CCUT_ERR_UNSUPPORTED;
  if (!L->w13 || !L->w2) return CCUT_ERR_INVALID;
  return CCUT_OK;
}

int check_route(const ccut_route_params* rp, int E) {
  if (!rp) return CCUT_ERR_INVALID;
  if (rp->top_k < 1 || rp->top_k > kMaxTopK || rp->top_k > E) return CCUT_ERR_INVALID;
  if (E > kMaxRoutedExperts) return CCUT_ERR_UNSUPPORTED;
  if (rp->mode == CCUT_ROUTE_SIGMOID_GROUP) {
    if (rp->n_group < 1 || rp->n_group > 32 || E % rp->n_group) return CCUT_ERR_INVALID;
    if (rp->topk_group < 1 || rp->topk_group > rp->n_group) return CCUT_ERR_INVALID;
    if (rp->topk_group * (E / rp->n_group) < rp->top_k) return CCUT_ERR_INVALID;
  } else if (rp->mode != CCUT_ROUTE_SOFTMAX_TOPK && rp->mode != CCUT_ROUTE_TOPK_SOFTMAX) {
    return CCUT_ERR_UNSUPPORTED;
  }
  return CCUT_OK;
}

// Token-tile height of the mma.sync kernel from the mean rows per routed expert.
// CCUT_MMA_TOKEN_TILE (16, 32 or 64) overrides it, for measurement.
int pick_mt(long rows_per_expert) {
  static const int forced = [] {
    const char* v = getenv("CCUT_MMA_TOKEN_TILE");
    const int t = v ? atoi(v) : 0;
    return (t == 16 || t == 32 || t == 64) ? t : 0;
  }();
  if (forced) return forced;
  return rows_per_expert <= 10 ? 16 : rows_per_expert <= 24 ? 32 : 64;
}

// Kernel choice for a call with T tokens and top_k k.
long mean_rows(const ccut_moe_layer* L, int T, int k) {
  return (long)T * k / (L->num_experts > 0 ? L->num_experts : 1);
}

bool use_tc(const ccut_moe_layer* L, long per_expert) {
  if (L->kernel == CCUT_KERNEL_TC) return true;
  if (L->kernel == CCUT_KERNEL_MMA) return false;
  if (!L->w13_frags || !L->w2_frags) return true;
  return per_expert >= CCUT_TC_MIN_ROWS;
}

size_t rows_of(const ccut_moe_layer* L, int T, int k) { return (size_t)T * k + (size_t)L->num_shared_slices * T; }

FfnScratch carve_ffn(Carver& c, const ccut_moe_layer* L, int T, int k, bool with_input, int* sched) {
  const size_t R = rows_of(L, T, k);
  FfnScratch s{nullptr, nullptr, nullptr, sched};
  if (with_input) {  // sized for either kernel so that one workspace serves both
    s.xp = c.take<uint16_t>(R * L->hidden);
    s.x16 = c.take<uint16_t>((size_t)T * L->hidden);
  }
  s.hbuf = c.take<uint16_t>(R * L->inter);
  return s;
}

// Work counters of a mma.sync launch (static schedule when null).
// CCUT_DYNAMIC_SCHEDULE=0 selects the static schedule, for measurement.
static void set_sched(GemmArgs& a, int* sched) {
  static const bool off = [] {
    const char* v = getenv("CCUT_DYNAMIC_SCHEDULE");
    return v && v[0] == '0';
  }();
  a.sched = off ? nullptr : sched;
}

struct FwdScratch {
  int* status;
  int* sched;
  float* part;
  int* counts;
  int32_t* offsets;
  int32_t* ids;
  float* wts;
  int32_t* row_token;
  float* row_weight;
  int32_t* pair_row;
  FfnScratch ffn;
  float* ybuf;
};

FwdScratch carve_fwd(Carver& c, const ccut_moe_layer* L, int T, int k) {
  const int E = L->num_experts, H = L->hidden, S = L->num_shared_slices;
  const size_t R = (size_t)T * k + (size_t)S * T;
  FwdScratch s;
  s.status = c.take<int>(64);
  s.sched = take_sched(c);
  s.part = c.take<float>((size_t)route_scratch_floats(T, E, H));
  s.counts = c.take<int>(E);
  s.offsets = c.take<int32_t>(E + S + 1);
  s.ids = c.take<int32_t>((size_t)T * k);
  s.wts = c.take<float>((size_t)T * k);
  s.row_token = c.take<int32_t>(R);
  s.row_weight = c.take<float>(R);
  s.pair_row = c.take<int32_t>((size_t)T * k);
  s.ffn = carve_ffn(c, L, T, k, true, s.sched);
  s.ybuf = c.take<float>(R * H);
  return s;
}


// gate/up: h rows [R, I] from x: bf16 from the tcgen05 kernel, f16 from the mma.sync kernel
// (run_down reads them with the same kernel).  `x16` is the mma.sync path's f16 copy of x;
// `xp` the tcgen05 path's bf16 gather buffer.
int run_gate_up(const ccut_moe_layer* L, long per_expert, const uint16_t* x, const uint16_t* x16, uint16_t* xp,
                int T, int k, const int32_t* offsets, const int32_t* row_token, uint16_t* hbuf, int* sched, int* status,
                cudaStream_t st) {
  const int fmt = L->format;
  const int ne = L->num_experts + L->num_shared_slices;
  if (use_tc(L, per_expert)) {
    const int R = static_cast<int>(rows_of(L, T, k));
    int rc = launch_gather_rows(x, row_token, R, offsets + ne, L->hidden, xp, st);
    if (rc) return rc;
    CUtensorMap map;
    rc = encode_rows_map(&map, xp, R, L->hidden, kTcBoxRows);
    if (rc) return rc;
    // fused gate/up rows: 2I packed rows, intermediate rows of I channels out
    TcArgs a{static_cast<const uint8_t*>(L->w13), ccut_w13_bytes(fmt, L->hidden, L->inter), L->hidden,
             2 * L->inter, offsets, ne, hbuf, L->inter, nullptr, status};
    a.sched = sched;
    return launch_tc_gemm(fmt, kFfn1, map, a, num_sms(), st);
  }
  if (!x16) return CCUT_ERR_INVALID;
  GemmArgs a{static_cast<const uint8_t*>(L->w13_frags),
             ccut_w13_bytes(fmt, L->hidden, L->inter),
             L->hidden,
             L->inter,
             x16,
             L->hidden,
             row_token,
             offsets,
             ne,
             hbuf,
             L->inter,
             nullptr,
             status};
  set_sched(a, sched);
  return launch_gemm(fmt, kFfn1, pick_mt(per_expert), a, num_sms(), st);
}

// down: weighted rows y [R, H], fp32 or (y_bf16) bf16.
int run_down(const ccut_moe_layer* L, long per_expert, const uint16_t* hbuf, int T, int k, const int32_t* offsets,
             const float* row_weight, void* y_rows, int y_bf16, int* sched, int* status, cudaStream_t st) {
  const int fmt = L->format;
  const int ne = L->num_experts + L->num_shared_slices;
  if (use_tc(L, per_expert)) {
    const int R = static_cast<int>(rows_of(L, T, k));
    CUtensorMap map;
    int rc = encode_rows_map(&map, hbuf, R, L->inter, kTcBoxRows);
    if (rc) return rc;
    TcArgs a{static_cast<const uint8_t*>(L->w2), ccut_w2_bytes(fmt, L->hidden, L->inter), L->inter, L->hidden,
             offsets, ne, y_rows, L->hidden, row_weight, status, y_bf16};
    a.sched = sched;
    return launch_tc_gemm(fmt, kFfn2, map, a, num_sms(), st);
  }
  GemmArgs a{static_cast<const uint8_t*>(L->w2_frags),
             ccut_w2_bytes(fmt, L->hidden, L->inter),
             L->inter,
             L->hidden,
             hbuf,
             L->inter,
             nullptr,
             offsets,
             ne,
             y_rows,
             L->hidden,
             row_weight,
             status};
  a.out_bf16 = y_bf16;
  set_sched(a, sched);
  return launch_gemm(fmt, kFfn2, pick_mt(per_expert), a, num_sms(), st);
}

int run_ffn(const ccut_moe_layer* L, long per_expert, const uint16_t* x, const FfnScratch& s, int T, int k,
            const int32_t* offsets, const int32_t* row_token, const float* row_weight, void* y_rows, int y_bf16,
            int* status, cudaStream_t st) {
  int rc = run_gate_up(L, per_expert, x, s.x16, s.xp, T, k, offsets, row_token, s.hbuf, s.sched, status, st);
  if (rc) return rc;
  return run_down(L, per_expert, s.hbuf, T, k, offsets, row_weight, y_rows, y_bf16, s.sched, status, st);
}

// The bounded waits of the kernels, exercised on barriers with a known outcome: barrier 0
// completes (one arrival), barrier 1 never does (nothing arrives on it).  Both wait forms
// run out on barrier 1 after `budget` cycles and record CCUT_ERR_TIMEOUT in the status word;
// the kernel then returns.
__global__ void wait_expiry_kernel(int* status, long long budget, int* outcome) {
  __shared__ uint64_t bars[2];
  if (threadIdx.x == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    mbar_arrive(&bars[0]);
    const bool done = mbar_wait(&bars[0], 0, status, budget);            // completes
    const bool late = mbar_wait(&bars[1], 0, status, budget);            // runs out
    const bool late_spin = mbar_spin(&bars[1], 0, status, budget);       // runs out
    outcome[0] = (done ? 1 : 0) | (late ? 2 : 0) | (late_spin ? 4 : 0);
  }
}

}  // namespace ccut

using namespace ccut;

extern "C" {

int ccut_debug_wait_expiry(void* workspace, long long budget_cycles, ccut_stream_t stream) {
  if (!workspace || budget_cycles < 0 || budget_cycles > kWaitBudgetCycles) return CCUT_ERR_INVALID;
  int* ws = static_cast<int*>(workspace);
  // outcome flags at ws[1]: bit 0 = the completed barrier's wait succeeded, bits 1-2 = the
  // waits on the barrier nothing arrives on succeeded (both stay 0)
  return launch_k(wait_expiry_kernel, dim3(1), dim3(32), 0, stream, ws, budget_cycles, ws + 1);
}

const char* ccut_strerror(int code) {
  switch (code) {
    case CCUT_OK: return "ok";
    case CCUT_ERR_INVALID: return "invalid argument or shape";
    case CCUT_ERR_UNSUPPORTED: return "unsupported format, mode or size";
    case CCUT_ERR_CUDA: return "CUDA launch or runtime failure";
    case CCUT_ERR_WORKSPACE: return "workspace too small";
    case CCUT_ERR_TIMEOUT: return "bounded device wait expired";
    case CCUT_ERR_NCCL: return "NCCL failure";
    default: return "unknown error";
  }
}

int ccut_abi_version(void) { return 1; }

size_t ccut_packed_matrix_bytes(int format, int K, int N) {
  if (!valid_fmt(format) || K <= 0 || N <= 0 || K % 128 || N % 128) return 0;
  return (size_t)(N / kTileN) * (K / kTileK) * block_bytes(format);
}

size_t ccut_w13_bytes(int format, int hidden, int inter) { return 2 * ccut_packed_matrix_bytes(format, hidden, inter); }

size_t ccut_w2_bytes(int format, int hidden, int inter) { return ccut_packed_matrix_bytes(format, inter, hidden); }

int ccut_pack_matrix(int format, int layout, const void* q, const void* z, const void* s, int K, int N,
                     int nibble_order, void* dst, int nmat, int slot, ccut_stream_t stream) {
  if (!valid_fmt(format)) return CCUT_ERR_UNSUPPORTED;
  if (layout != CCUT_LAYOUT_ROWS && layout != CCUT_LAYOUT_FRAGS) return CCUT_ERR_UNSUPPORTED;
  if (!q || !s || !dst || K <= 0 || N <= 0 || K % 128 || N % 128) return CCUT_ERR_INVALID;
  if (nmat < 1 || nmat > 2 || slot < 0 || slot >= nmat) return CCUT_ERR_INVALID;
  if (format == CCUT_FMT_AWQ_INT4_G128 && !z) return CCUT_ERR_INVALID;
  if ((format == CCUT_FMT_AWQ_INT4_G128 || format == CCUT_FMT_INT4_SYM_G128) &&
      nibble_order != CCUT_NIBBLES_AWQ && nibble_order != CCUT_NIBBLES_SEQUENTIAL)
    return CCUT_ERR_INVALID;
  return launch_pack(format, layout, q, z, s, K, N, nibble_order, dst, nmat, slot, stream);
}

int ccut_dequant_matrix(int format, int layout, const void* packed, int K, int N, int nmat, int slot, float* out,
                        ccut_stream_t stream) {
  if (!valid_fmt(format)) return CCUT_ERR_UNSUPPORTED;
  if (layout != CCUT_LAYOUT_ROWS && layout != CCUT_LAYOUT_FRAGS) return CCUT_ERR_UNSUPPORTED;
  if (!packed || !out || K <= 0 || N <= 0 || K % 128 || N % 128) return CCUT_ERR_INVALID;
  if (nmat < 1 || nmat > 2 || slot < 0 || slot >= nmat) return CCUT_ERR_INVALID;
  return launch_dequant(format, layout, packed, K, N, nmat, slot, out, stream);
}

size_t ccut_route_workspace_bytes(int T, int E, int H) {
  if (T <= 0 || E <= 0 || H <= 0 || H % 64) return 256;
  Carver c(nullptr);
  c.take<int>(64);
  c.take<float>((size_t)route_scratch_floats(T, E, H));
  return c.off;
}

int ccut_moe_route(const uint16_t* x, const float* router, int T, int H, int E, const ccut_route_params* rp,
                   int32_t* ids, float* weights, float* logits, void* workspace, size_t ws_bytes,
                   ccut_stream_t stream) {
  PdlScope pdl_scope(T);  // PDL for decode-sized calls
  int rc = check_route(rp, E);
  if (rc) return rc;
  if (T < 0 || H <= 0 || H % 128) return CCUT_ERR_INVALID;
  if (T == 0) return CCUT_OK;
  if (!x || !router || !ids || !weights || !workspace) return CCUT_ERR_INVALID;
  if (ws_bytes < ccut_route_workspace_bytes(T, E, H)) return CCUT_ERR_WORKSPACE;
  Carver c(workspace);
  c.take<int>(64);
  float* part = c.take<float>((size_t)route_scratch_floats(T, E, H));
  return launch_route(x, router, T, H, E, *rp, ids, weights, logits, part, nullptr, nullptr, stream);
}

int ccut_moe_topk(const float* logits, int T, int E, const ccut_route_params* rp, int32_t* ids, float* weights,
                  ccut_stream_t stream) {
  PdlScope pdl_scope(T);  // PDL for decode-sized calls
  int rc = check_route(rp, E);
  if (rc) return rc;
  if (T < 0) return CCUT_ERR_INVALID;
  if (T == 0) return CCUT_OK;
  if (!logits || !ids || !weights) return CCUT_ERR_INVALID;
  return launch_topk(logits, T, E, *rp, ids, weights, stream);
}

size_t ccut_permute_workspace_bytes(int E) {
  Carver c(nullptr);
  c.take<int>(64);
  c.take<int>(E > 0 ? E : 1);
  return c.off;
}

int ccut_moe_permute(const int32_t* ids, const float* weights, int T, int k, int E, int num_shared_slices,
                     float shared_gate, int32_t* offsets, int32_t* row_token, float* row_weight, int32_t* pair_row,
                     void* workspace, size_t ws_bytes, ccut_stream_t stream) {
  PdlScope pdl_scope(T);  // PDL for decode-sized calls
  if (T < 0 || k < 1 || k > kMaxTopK || E < 1 || E > kMaxRoutedExperts || num_shared_slices < 0 ||
      E + num_shared_slices > kMaxExperts)
    return CCUT_ERR_INVALID;
  if (!offsets || !row_token || !row_weight || !pair_row || !workspace || (T > 0 && (!ids || !weights)))
    return CCUT_ERR_INVALID;
  if (ws_bytes < ccut_permute_workspace_bytes(E)) return CCUT_ERR_WORKSPACE;
  Carver c(workspace);
  c.take<int>(64);
  int* counts = c.take<int>(E);
  int rc = launch_count(ids, T * k, E, counts, stream);
  if (rc) return rc;
  return launch_permute(ids, weights, T, k, E, num_shared_slices, shared_gate, counts, offsets, row_token,
                        row_weight, pair_row, stream);
}

size_t ccut_expert_ffn_workspace_bytes(const ccut_moe_layer* L, int T, int k) {
  if (check_layer(L) || T < 0 || k < 1) return 0;
  Carver c(nullptr);
  c.take<int>(64);
  take_sched(c);
  carve_ffn(c, L, T, k, true, nullptr);
  return c.off;
}

int ccut_moe_expert_ffn(const ccut_moe_layer* L, const uint16_t* x, int T, int k, const int32_t* offsets,
                        const int32_t* row_token, const float* row_weight, float* y_rows, void* workspace,
                        size_t ws_bytes, ccut_stream_t stream) {
  PdlScope pdl_scope(T);  // PDL for decode-sized calls
  int rc = check_layer(L);
  if (rc) return rc;
  if (T < 0 || k < 1 || k > kMaxTopK || k > L->num_experts) return CCUT_ERR_INVALID;
  if (T == 0) return CCUT_OK;
  if (!x || !offsets || !row_token || !row_weight || !y_rows || !workspace) return CCUT_ERR_INVALID;
  if (ws_bytes < ccut_expert_ffn_workspace_bytes(L, T, k)) return CCUT_ERR_WORKSPACE;
  Carver c(workspace);
  int* status = c.take<int>(64);
  int* sched = take_sched(c);
  FfnScratch s = carve_ffn(c, L, T, k, true, sched);
  if (s.x16 && !use_tc(L, mean_rows(L, T, k))) {
    rc = launch_bf16_to_f16(x, s.x16, (size_t)T * L->hidden, stream);
    if (rc) return rc;
  }
  return run_ffn(L, mean_rows(L, T, k), x, s, T, k, offsets, row_token, row_weight, y_rows, 0, status, stream);
}

int ccut_moe_expert_ffn_w4a16(const ccut_moe_layer* L, const uint16_t* x, int T, int k, const int32_t* offsets,
                              const int32_t* row_token, const float* row_weight, float* y_rows, void* workspace,
                              size_t ws_bytes, ccut_stream_t stream) {
  if (!L || (L->format != CCUT_FMT_AWQ_INT4_G128 && L->format != CCUT_FMT_INT4_SYM_G128)) return CCUT_ERR_UNSUPPORTED;
  return ccut_moe_expert_ffn(L, x, T, k, offsets, row_token, row_weight, y_rows, workspace, ws_bytes, stream);
}

int ccut_moe_expert_ffn_fp8b128(const ccut_moe_layer* L, const uint16_t* x, int T, int k, const int32_t* offsets,
                                const int32_t* row_token, const float* row_weight, float* y_rows, void* workspace,
                                size_t ws_bytes, ccut_stream_t stream) {
  if (!L || L->format != CCUT_FMT_FP8_E4M3_B128) return CCUT_ERR_UNSUPPORTED;
  return ccut_moe_expert_ffn(L, x, T, k, offsets, row_token, row_weight, y_rows, workspace, ws_bytes, stream);
}

int ccut_moe_expert_ffn_w8a16(const ccut_moe_layer* L, const uint16_t* x, int T, int k, const int32_t* offsets,
                              const int32_t* row_token, const float* row_weight, float* y_rows, void* workspace,
                              size_t ws_bytes, ccut_stream_t stream) {
  if (!L || L->format != CCUT_FMT_FP8_E4M3_CH) return CCUT_ERR_UNSUPPORTED;
  return ccut_moe_expert_ffn(L, x, T, k, offsets, row_token, row_weight, y_rows, workspace, ws_bytes, stream);
}

size_t ccut_gate_up_workspace_bytes(const ccut_moe_layer* L, int T) {
  if (check_layer(L) || T < 0) return 0;
  Carver c(nullptr);
  c.take<int>(64);
  take_sched(c);
  // sized for the largest top_k and either kernel so that one workspace serves any call
  c.take<uint16_t>(rows_of(L, T, kMaxTopK) * L->hidden);
  c.take<uint16_t>((size_t)T * L->hidden);
  return c.off;
}

int ccut_moe_gate_up(const ccut_moe_layer* L, const uint16_t* x, int T, int k, const int32_t* offsets,
                     const int32_t* row_token, uint16_t* h_rows, void* workspace, size_t ws_bytes,
                     ccut_stream_t stream) {
  PdlScope pdl_scope(T);  // PDL for decode-sized calls
  int rc = check_layer(L);
  if (rc) return rc;
  if (T < 0 || k < 1 || k > kMaxTopK || k > L->num_experts) return CCUT_ERR_INVALID;
  if (T == 0) return CCUT_OK;
  if (!x || !offsets || !row_token || !h_rows || !workspace) return CCUT_ERR_INVALID;
  if (ws_bytes < ccut_gate_up_workspace_bytes(L, T)) return CCUT_ERR_WORKSPACE;
  Carver c(workspace);
  int* status = c.take<int>(64);
  int* sched = take_sched(c);
  uint16_t* xp = c.take<uint16_t>(rows_of(L, T, kMaxTopK) * L->hidden);
  uint16_t* x16 = c.take<uint16_t>((size_t)T * L->hidden);
  if (!use_tc(L, mean_rows(L, T, k))) {
    rc = launch_bf16_to_f16(x, x16, (size_t)T * L->hidden, stream);
    if (rc) return rc;
  }
  return run_gate_up(L, mean_rows(L, T, k), x, x16, xp, T, k, offsets, row_token, h_rows, sched, status, stream);
}

size_t ccut_down_workspace_bytes(const ccut_moe_layer* L) {
  if (check_layer(L)) return 0;
  Carver c(nullptr);
  c.take<int>(64);
  take_sched(c);
  return c.off;
}

int ccut_moe_down(const ccut_moe_layer* L, const uint16_t* h_rows, int T, int k, const int32_t* offsets,
                  const float* row_weight, float* y_rows, void* workspace, size_t ws_bytes, ccut_stream_t stream) {
  PdlScope pdl_scope(T);  // PDL for decode-sized calls
  int rc = check_layer(L);
  if (rc) return rc;
  if (T < 0 || k < 1 || k > kMaxTopK || k > L->num_experts) return CCUT_ERR_INVALID;
  if (T == 0) return CCUT_OK;
  if (!h_rows || !offsets || !row_weight || !y_rows || !workspace) return CCUT_ERR_INVALID;
  if (ws_bytes < 256) return CCUT_ERR_WORKSPACE;
  int* sched = nullptr;
  if (ws_bytes >= ccut_down_workspace_bytes(L)) {  // else the static schedule (status word only)
    Carver c(workspace);
    c.take<int>(64);
    sched = take_sched(c);
  }
  return run_down(L, mean_rows(L, T, k), h_rows, T, k, offsets, row_weight, y_rows, 0, sched,
                  static_cast<int*>(workspace), stream);
}

int ccut_moe_combine(const float* y_rows, const int32_t* pair_row, int T, int k, int H, int num_shared_slices,
                     void* out, int out_dtype, ccut_stream_t stream) {
  PdlScope pdl_scope(T);  // PDL for decode-sized calls
  if (T < 0 || k < 1 || k > kMaxTopK || H <= 0 || H % 4 || num_shared_slices < 0) return CCUT_ERR_INVALID;
  if (num_shared_slices > CCUT_MAX_SHARED_SLICES) return CCUT_ERR_UNSUPPORTED;
  if (out_dtype != CCUT_OUT_BF16 && out_dtype != CCUT_OUT_F32) return CCUT_ERR_INVALID;
  if (T == 0) return CCUT_OK;
  if (!y_rows || !pair_row || !out) return CCUT_ERR_INVALID;
  return launch_combine(y_rows, 0, pair_row, T, k, H, num_shared_slices, -1, out, out_dtype, stream);
}

size_t ccut_moe_forward_workspace_bytes(const ccut_moe_layer* L, int T, int top_k) {
  if (check_layer(L) || T < 0 || top_k < 1) return 0;
  if (T == 0) return 256;
  Carver c(nullptr);
  carve_fwd(c, L, T, top_k);
  return c.off;
}

int ccut_moe_forward(const ccut_moe_layer* L, const ccut_route_params* rp, const uint16_t* x, int T, void* out,
                     int out_dtype, int32_t* ids, float* weights, void* workspace, size_t ws_bytes,
                     ccut_stream_t stream) {
  PdlScope pdl_scope(T);  // PDL for decode-sized calls
  int rc = check_layer(L);
  if (rc) return rc;
  if (!L->router) return CCUT_ERR_INVALID;
  rc = check_route(rp, L->num_experts);
  if (rc) return rc;
  if (out_dtype != CCUT_OUT_BF16 && out_dtype != CCUT_OUT_F32) return CCUT_ERR_INVALID;
  if (T < 0) return CCUT_ERR_INVALID;
  if (T == 0) return CCUT_OK;
  if (!x || !out || !workspace) return CCUT_ERR_INVALID;
  const int k = rp->top_k, E = L->num_experts, H = L->hidden;
  if (ws_bytes < ccut_moe_forward_workspace_bytes(L, T, k)) return CCUT_ERR_WORKSPACE;
  Carver c(workspace);
  FwdScratch s = carve_fwd(c, L, T, k);
  cudaStream_t st = stream;
  rc = launch_route(x, L->router, T, H, E, *rp, s.ids, s.wts, nullptr, s.part, s.counts,
                    use_tc(L, mean_rows(L, T, k)) ? nullptr : s.ffn.x16, st);  // x16: mma.sync operands
  if (rc) return rc;
  rc = launch_permute(s.ids, s.wts, T, k, E, L->num_shared_slices, L->shared_gate, s.counts, s.offsets, s.row_token,
                      s.row_weight, s.pair_row, st);
  if (rc) return rc;
  // bf16 output: the weighted rows go through bf16 (one rounding each, half the bytes of
  // the down GEMM's writes and the combine's reads); fp32 output keeps fp32 rows
  const int y_bf16 = out_dtype == CCUT_OUT_BF16;
  rc = run_ffn(L, mean_rows(L, T, k), x, s.ffn, T, k, s.offsets, s.row_token, s.row_weight, s.ybuf, y_bf16, s.status,
               st);
  if (rc) return rc;
  rc = launch_combine(s.ybuf, y_bf16, s.pair_row, T, k, H, L->num_shared_slices, -1, out, out_dtype, st);
  if (rc) return rc;
  if (ids && cudaMemcpyAsync(ids, s.ids, sizeof(int32_t) * (size_t)T * k, cudaMemcpyDeviceToDevice, st) != cudaSuccess)
    return CCUT_ERR_CUDA;
  if (weights &&
      cudaMemcpyAsync(weights, s.wts, sizeof(float) * (size_t)T * k, cudaMemcpyDeviceToDevice, st) != cudaSuccess)
    return CCUT_ERR_CUDA;
  return CCUT_OK;
}

size_t ccut_quant_linear_workspace_bytes(int format, int M, int K) {
  if (!valid_fmt(format) || M < 0 || K <= 0) return 0;
  Carver c(nullptr);
  c.take<int>(64);
  c.take<int32_t>(2);
  c.take<uint16_t>((size_t)(M > 0 ? M : 1) * K);  // f16 activations
  return c.off;
}

int ccut_quant_linear(int format, int layout, const void* packed, int K, int N, const uint16_t* x, int M, float* y,
                      void* workspace, size_t ws_bytes, ccut_stream_t stream) {
  PdlScope pdl_scope(M);  // PDL for decode-sized calls
  if (!valid_fmt(format)) return CCUT_ERR_UNSUPPORTED;
  if (layout != CCUT_LAYOUT_ROWS && layout != CCUT_LAYOUT_FRAGS) return CCUT_ERR_UNSUPPORTED;
  if (K <= 0 || N <= 0 || K % 128 || N % 128 || M < 0) return CCUT_ERR_INVALID;
  if (M == 0) return CCUT_OK;
  if (!packed || !x || !y || !workspace) return CCUT_ERR_INVALID;
  if (ws_bytes < ccut_quant_linear_workspace_bytes(format, M, K)) return CCUT_ERR_WORKSPACE;
  Carver c(workspace);
  int* status = c.take<int>(64);
  int32_t* off = c.take<int32_t>(2);
  uint16_t* x16 = c.take<uint16_t>((size_t)M * K);
  int rc = launch_fill_offsets(off, M, stream);
  if (rc) return rc;
  if (layout == CCUT_LAYOUT_ROWS) {  // x is already [M, K] bf16 rows: the TMA reads it in place
    CUtensorMap map;
    rc = encode_rows_map(&map, x, M, K, kTcBoxRows);
    if (rc) return rc;
    TcArgs a{static_cast<const uint8_t*>(packed), 0, K, N, off, 1, y, N, nullptr, status};
    return launch_tc_gemm(format, kFfn2, map, a, num_sms(), stream);
  }
  rc = launch_bf16_to_f16(x, x16, (size_t)M * K, stream);
  if (rc) return rc;
  GemmArgs a{static_cast<const uint8_t*>(packed), 0, K, N, x16, K, nullptr, off, 1, y, N, nullptr, status};
  return launch_gemm(format, kFfn2, M <= 16 ? 16 : M <= 32 ? 32 : 64, a, num_sms(), stream);
}

int ccut_workspace_status(void* workspace, ccut_stream_t stream) {
  if (!workspace) return CCUT_ERR_INVALID;
  int v = 0;
  if (cudaMemcpyAsync(&v, workspace, sizeof(int), cudaMemcpyDeviceToHost, stream) != cudaSuccess) return CCUT_ERR_CUDA;
  if (cudaStreamSynchronize(stream) != cudaSuccess) return CCUT_ERR_CUDA;
  if (v != 0 && cudaMemsetAsync(workspace, 0, sizeof(int), stream) != cudaSuccess) return CCUT_ERR_CUDA;
  return v;
}

}  // extern "C"
