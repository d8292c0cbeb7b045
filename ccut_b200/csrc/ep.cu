// ep.cu -- expert-parallel MoE forward, one process per GPU, over NCCL.
//
// Rank r of P holds the routed experts [expert_lo, expert_lo + E_r) plus every shared
// expert, and its own T_r tokens.  One forward:
//   1. route the local tokens against the global router (ids are global expert indices);
//   2. dispatch: one grouped NCCL all-gather of the tokens, ids and routing weights, so that
//      every rank sees all T = sum T_r tokens;
//   3. keep the (token, slot) pairs whose expert is local (others get id -1 and take no
//      row), permute them by local expert and run the grouped expert FFN on them only;
//   4. combine the local rows per token (fp32 [T, H], zero for tokens with no local
//      expert) and reduce-scatter it: rank r receives the sum over ranks of its T_r rows;
//   5. shared experts run data-parallel on the local tokens and are added in; they only need
//      the local tokens, so they run on a second stream while the dispatch is in flight.
// The reference runs the experts of one layer in a single process
// (ccut/models/generic.py:364-385, ccut/experts/pipeline.py:123-190); the partitioning is
// new.  One blocking NCCL communicator per layer handle carries the collectives.
#include <nccl.h>

#include <chrono>
#include <cstring>
#include <new>
#include <thread>

#include "host.cuh"

struct ccut_ep {
  ncclComm_t comm;
  int rank;
  int world;
  double timeout_s;
  cudaStream_t side;  // shared experts run here, beside the dispatch collective
  cudaEvent_t fork, join;
};

namespace ccut {
namespace {

// Wait (bounded) for a call on a non-blocking communicator to leave ncclInProgress.
int nccl_settle(ncclComm_t comm, ncclResult_t r, double budget_s) {
  const auto t0 = std::chrono::steady_clock::now();
  while (r == ncclInProgress) {
    if (std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count() > budget_s)
      return CCUT_ERR_TIMEOUT;
    std::this_thread::yield();
    if (ncclCommGetAsyncError(comm, &r) != ncclSuccess) return CCUT_ERR_NCCL;
  }
  return r == ncclSuccess ? CCUT_OK : CCUT_ERR_NCCL;
}

// ids_loc[i] = ids[i] - lo when expert ids[i] is local, else -1; weights copied; counts[e]
// of the local experts accumulated (shared-memory histogram, then one atomic per expert
// and CTA).  counts must start at zero.
__global__ void __launch_bounds__(256) localize_count_kernel(const int32_t* __restrict__ ids,
                                                             const float* __restrict__ w, int n, int lo, int e_local,
                                                             int32_t* __restrict__ ids_loc,
                                                             float* __restrict__ w_loc, int* __restrict__ counts) {
  pdl_wait();
  pdl_trigger();
  __shared__ int hist[kMaxExperts];
  for (int e = threadIdx.x; e < e_local; e += blockDim.x) hist[e] = 0;
  __syncthreads();
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const int e = ids[i] - lo;
    const bool mine = e >= 0 && e < e_local;
    ids_loc[i] = mine ? e : -1;
    w_loc[i] = w[i];
    if (mine) atomicAdd(&hist[e], 1);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < e_local; e += blockDim.x)
    if (hist[e]) atomicAdd(&counts[e], hist[e]);
}

// out = a (+ b), fp32 -> bf16 or fp32.
__global__ void add_cast_kernel(const float4* __restrict__ a, const float4* __restrict__ b, size_t n4, void* out,
                                int out_dtype) {
  pdl_wait();
  pdl_trigger();
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x) {
    float4 v = a[i];
    if (b) {
      const float4 u = b[i];
      v.x += u.x;
      v.y += u.y;
      v.z += u.z;
      v.w += u.w;
    }
    if (out_dtype == CCUT_OUT_BF16) {
      __nv_bfloat162 lo = __floats2bfloat162_rn(v.x, v.y), hi = __floats2bfloat162_rn(v.z, v.w);
      uint2 pk;
      pk.x = *reinterpret_cast<uint32_t*>(&lo);
      pk.y = *reinterpret_cast<uint32_t*>(&hi);
      static_cast<uint2*>(out)[i] = pk;
    } else {
      static_cast<float4*>(out)[i] = v;
    }
  }
}

int grid_for(size_t n, int per_block) {
  size_t b = (n + per_block - 1) / per_block;
  if (b > 148 * 8) b = 148 * 8;
  return b < 1 ? 1 : static_cast<int>(b);
}

// Layer views: the routed experts alone, and the shared slices behind one empty routed
// expert (the last local one, which receives no rows).
ccut_moe_layer routed_view(const ccut_moe_layer* L) {
  ccut_moe_layer v = *L;
  v.num_shared_slices = 0;
  return v;
}

ccut_moe_layer shared_view(const ccut_moe_layer* L) {
  ccut_moe_layer v = *L;
  const size_t o13 = ccut_w13_bytes(L->format, L->hidden, L->inter) * (size_t)(L->num_experts - 1);
  const size_t o2 = ccut_w2_bytes(L->format, L->hidden, L->inter) * (size_t)(L->num_experts - 1);
  auto adv = [](const void* p, size_t o) -> const void* {
    return p ? static_cast<const uint8_t*>(p) + o : nullptr;
  };
  v.num_experts = 1;
  v.w13 = adv(L->w13, o13);
  v.w2 = adv(L->w2, o2);
  v.w13_frags = adv(L->w13_frags, o13);
  v.w2_frags = adv(L->w2_frags, o2);
  return v;
}

// Kernel policy of a view for a mean of per_expert rows (unless the layer forces one).
ccut_moe_layer with_policy(ccut_moe_layer v, long per_expert) {
  if (v.kernel == CCUT_KERNEL_AUTO) v.kernel = use_tc(&v, per_expert) ? CCUT_KERNEL_TC : CCUT_KERNEL_MMA;
  return v;
}

struct EpScratch {
  int* status;
  int* sched;     // GEMM work counters of the routed FFN
  int* sh_sched;  // and of the shared-expert FFN (runs concurrently on the side stream)
  float* part;
  int* counts_g;
  int32_t* ids_l;
  float* w_l;
  uint16_t* x_all;
  int32_t* ids_all;
  float* w_all;
  int32_t* ids_loc;
  float* w_loc;
  int* counts;
  int32_t* offsets;
  int32_t* row_token;
  float* row_weight;
  int32_t* pair_row;
  FfnScratch ffn;
  float* ybuf;
  float* y_part;
  float* y_loc;
  // shared experts
  int32_t* sh_ids;
  float* sh_w;
  int* sh_counts;
  int32_t* sh_offsets;
  int32_t* sh_row_token;
  float* sh_row_weight;
  int32_t* sh_pair_row;
  FfnScratch sh_ffn;
  float* sh_ybuf;
  float* y_sh;
};

EpScratch carve_ep(Carver& c, const ccut_moe_layer* L, int E_global, int world, int T_l, int k) {
  const int H = L->hidden, S = L->num_shared_slices;
  const int T = world * T_l;
  const ccut_moe_layer rv = routed_view(L);
  EpScratch s{};
  s.status = c.take<int>(64);
  s.sched = take_sched(c);
  s.sh_sched = take_sched(c);
  s.part = c.take<float>((size_t)route_hsplit(T_l, E_global, H) * T_l * E_global);
  s.counts_g = c.take<int>(E_global);
  s.ids_l = c.take<int32_t>((size_t)T_l * k);
  s.w_l = c.take<float>((size_t)T_l * k);
  s.x_all = c.take<uint16_t>((size_t)T * H);
  s.ids_all = c.take<int32_t>((size_t)T * k);
  s.w_all = c.take<float>((size_t)T * k);
  s.ids_loc = c.take<int32_t>((size_t)T * k);
  s.w_loc = c.take<float>((size_t)T * k);
  s.counts = c.take<int>(L->num_experts);
  s.offsets = c.take<int32_t>(L->num_experts + 1);
  s.row_token = c.take<int32_t>((size_t)T * k);
  s.row_weight = c.take<float>((size_t)T * k);
  s.pair_row = c.take<int32_t>((size_t)T * k);
  s.ffn = carve_ffn(c, &rv, T, k, true, s.sched);
  s.ybuf = c.take<float>((size_t)T * k * H);
  s.y_part = c.take<float>((size_t)T * H);
  s.y_loc = c.take<float>((size_t)T_l * H);
  if (S > 0) {
    const ccut_moe_layer sv = shared_view(L);
    const size_t R = (size_t)(S + 1) * T_l;
    s.sh_ids = c.take<int32_t>(T_l);
    s.sh_w = c.take<float>(T_l);
    s.sh_counts = c.take<int>(1);
    s.sh_offsets = c.take<int32_t>(S + 2);
    s.sh_row_token = c.take<int32_t>(R);
    s.sh_row_weight = c.take<float>(R);
    s.sh_pair_row = c.take<int32_t>(T_l);
    s.sh_ffn = carve_ffn(c, &sv, T_l, 1, true, s.sh_sched);
    s.sh_ybuf = c.take<float>(R * H);
    s.y_sh = c.take<float>((size_t)T_l * H);
  }
  return s;
}

int check_ep(const ccut_ep* ep) {
  if (!ep || !ep->comm || ep->world < 1 || ep->rank < 0 || ep->rank >= ep->world) return CCUT_ERR_INVALID;
  return CCUT_OK;
}

int ep_allgather(ccut_ep* ep, const uint16_t* x, const int32_t* ids, const float* w, int T_l, int H, int k,
                 uint16_t* x_all, int32_t* ids_all, float* w_all, cudaStream_t st) {
  ncclResult_t r = ncclGroupStart();
  if (r != ncclSuccess) return CCUT_ERR_NCCL;
  ncclAllGather(x, x_all, (size_t)T_l * H * 2, ncclUint8, ep->comm, st);
  ncclAllGather(ids, ids_all, (size_t)T_l * k, ncclInt32, ep->comm, st);
  ncclAllGather(w, w_all, (size_t)T_l * k, ncclFloat32, ep->comm, st);
  return nccl_settle(ep->comm, ncclGroupEnd(), ep->timeout_s);
}

int ep_reduce_scatter(ccut_ep* ep, const float* y_part, int T_l, int H, float* y_loc, cudaStream_t st) {
  return nccl_settle(ep->comm,
                     ncclReduceScatter(y_part, y_loc, (size_t)T_l * H, ncclFloat32, ncclSum, ep->comm, st),
                     ep->timeout_s);
}

}  // namespace
}  // namespace ccut

using namespace ccut;

extern "C" {

size_t ccut_ep_unique_id_bytes(void) { return sizeof(ncclUniqueId); }

int ccut_ep_unique_id(void* id_out) {
  if (!id_out) return CCUT_ERR_INVALID;
  ncclUniqueId id;
  if (ncclGetUniqueId(&id) != ncclSuccess) return CCUT_ERR_NCCL;
  std::memcpy(id_out, &id, sizeof(id));
  return CCUT_OK;
}

int ccut_ep_init(const void* unique_id, int rank, int world, double timeout_s, ccut_ep** out) {
  if (!unique_id || !out || world < 1 || rank < 0 || rank >= world || !(timeout_s > 0)) return CCUT_ERR_INVALID;
  *out = nullptr;
  ncclUniqueId id;
  std::memcpy(&id, unique_id, sizeof(id));
  // A blocking communicator: init returns once every rank has joined (the caller bounds
  // that wait: the unique id reaches the ranks through a collective with a timeout, and the
  // process has its own limit); collectives are enqueued without host polling.
  ncclComm_t comm = nullptr;
  if (ncclCommInitRank(&comm, world, id, rank) != ncclSuccess) {
    if (comm) ncclCommAbort(comm);
    return CCUT_ERR_NCCL;
  }
  ccut_ep* ep = new (std::nothrow) ccut_ep{comm, rank, world, timeout_s, nullptr, nullptr, nullptr};
  if (!ep) {
    ncclCommAbort(comm);
    return CCUT_ERR_INVALID;
  }
  if (cudaStreamCreateWithFlags(&ep->side, cudaStreamNonBlocking) != cudaSuccess ||
      cudaEventCreateWithFlags(&ep->fork, cudaEventDisableTiming) != cudaSuccess ||
      cudaEventCreateWithFlags(&ep->join, cudaEventDisableTiming) != cudaSuccess) {
    ccut_ep_destroy(ep);
    return CCUT_ERR_CUDA;
  }
  *out = ep;
  return CCUT_OK;
}

int ccut_ep_destroy(ccut_ep* ep) {
  if (!ep) return CCUT_OK;
  int rc = CCUT_OK;
  if (ep->comm) {
    rc = nccl_settle(ep->comm, ncclCommFinalize(ep->comm), ep->timeout_s);
    if (rc == CCUT_OK) {
      rc = nccl_settle(ep->comm, ncclCommDestroy(ep->comm), ep->timeout_s);
    } else {
      ncclCommAbort(ep->comm);
    }
  }
  if (ep->side) cudaStreamDestroy(ep->side);
  if (ep->fork) cudaEventDestroy(ep->fork);
  if (ep->join) cudaEventDestroy(ep->join);
  delete ep;
  return rc;
}

int ccut_moe_ep_dispatch(ccut_ep* ep, const uint16_t* x, const int32_t* ids, const float* weights, int T_local,
                         int H, int k, uint16_t* x_all, int32_t* ids_all, float* w_all, ccut_stream_t stream) {
  int rc = check_ep(ep);
  if (rc) return rc;
  if (T_local < 0 || H <= 0 || k < 1 || k > kMaxTopK) return CCUT_ERR_INVALID;
  if (T_local == 0) return CCUT_OK;
  if (!x || !ids || !weights || !x_all || !ids_all || !w_all) return CCUT_ERR_INVALID;
  return ep_allgather(ep, x, ids, weights, T_local, H, k, x_all, ids_all, w_all, stream);
}

int ccut_moe_ep_combine(ccut_ep* ep, const float* y_part, int T_local, int H, float* y_local, ccut_stream_t stream) {
  int rc = check_ep(ep);
  if (rc) return rc;
  if (T_local < 0 || H <= 0) return CCUT_ERR_INVALID;
  if (T_local == 0) return CCUT_OK;
  if (!y_part || !y_local) return CCUT_ERR_INVALID;
  return ep_reduce_scatter(ep, y_part, T_local, H, y_local, stream);
}

size_t ccut_moe_ep_forward_workspace_bytes(const ccut_moe_layer* L, int num_experts_global, int world,
                                           int T_local, int top_k) {
  if (check_layer(L) || world < 1 || T_local < 0 || top_k < 1 || num_experts_global < L->num_experts) return 0;
  Carver c(nullptr);
  carve_ep(c, L, num_experts_global, world, T_local, top_k);
  return c.off;
}

int ccut_moe_ep_forward(ccut_ep* ep, const ccut_moe_layer* L, int expert_lo, int num_experts_global,
                        const ccut_route_params* rp, const uint16_t* x, int T_local, void* out, int out_dtype,
                        void* workspace, size_t ws_bytes, ccut_stream_t stream) {
  int rc = check_ep(ep);
  if (rc) return rc;
  PdlScope pdl_scope((long)T_local * ep->world);  // PDL for decode-sized calls (all ranks' tokens)
  rc = check_layer(L);
  if (rc) return rc;
  if (!L->router) return CCUT_ERR_INVALID;
  if (num_experts_global < 1 || num_experts_global > kMaxRoutedExperts || expert_lo < 0 ||
      expert_lo + L->num_experts > num_experts_global)
    return CCUT_ERR_INVALID;
  rc = check_route(rp, num_experts_global);
  if (rc) return rc;
  if (out_dtype != CCUT_OUT_BF16 && out_dtype != CCUT_OUT_F32) return CCUT_ERR_INVALID;
  if (T_local < 0) return CCUT_ERR_INVALID;
  // every rank must take part in the collectives, so an empty local batch still runs them
  const int k = rp->top_k, H = L->hidden, E_l = L->num_experts, S = L->num_shared_slices;
  const int T = ep->world * T_local;
  if (T_local > 0 && (!x || !out)) return CCUT_ERR_INVALID;
  if (!workspace) return CCUT_ERR_INVALID;
  if (ws_bytes < ccut_moe_ep_forward_workspace_bytes(L, num_experts_global, ep->world, T_local, k))
    return CCUT_ERR_WORKSPACE;
  if (T == 0) return CCUT_OK;
  cudaStream_t st = stream;
  Carver c(workspace);
  EpScratch s = carve_ep(c, L, num_experts_global, ep->world, T_local, k);

  // 5 (forked). shared experts on the local tokens, on the side stream: no routed pair is
  //    valid there, so every row belongs to a shared slice (rows s * T_local + t)
  const bool shared = S > 0 && T_local > 0;
  if (shared) {
    cudaStream_t ss = ep->side;
    if (cudaEventRecord(ep->fork, st) != cudaSuccess || cudaStreamWaitEvent(ss, ep->fork, 0) != cudaSuccess)
      return CCUT_ERR_CUDA;
    if (cudaMemsetAsync(s.sh_ids, 0xFF, sizeof(int32_t) * T_local, ss) != cudaSuccess) return CCUT_ERR_CUDA;
    if (cudaMemsetAsync(s.sh_pair_row, 0xFF, sizeof(int32_t) * T_local, ss) != cudaSuccess) return CCUT_ERR_CUDA;
    if (cudaMemsetAsync(s.sh_counts, 0, sizeof(int), ss) != cudaSuccess) return CCUT_ERR_CUDA;
    rc = launch_permute(s.sh_ids, s.sh_w, T_local, 1, 1, S, L->shared_gate, s.sh_counts, s.sh_offsets,
                        s.sh_row_token, s.sh_row_weight, s.sh_pair_row, ss);
    if (rc) return rc;
    const ccut_moe_layer sv = with_policy(shared_view(L), T_local);
    if (sv.kernel == CCUT_KERNEL_MMA) {
      rc = launch_bf16_to_f16(x, s.sh_ffn.x16, (size_t)T_local * H, ss);
      if (rc) return rc;
    }
    rc = run_ffn(&sv, T_local, x, s.sh_ffn, T_local, 1, s.sh_offsets, s.sh_row_token, s.sh_row_weight, s.sh_ybuf,
                 s.status, ss);
    if (rc) return rc;
    rc = launch_combine(s.sh_ybuf, s.sh_pair_row, T_local, 1, H, S, 0, s.y_sh, CCUT_OUT_F32, ss);
    if (rc) return rc;
    if (cudaEventRecord(ep->join, ss) != cudaSuccess) return CCUT_ERR_CUDA;
  }
  // 1. route the local tokens (global expert ids)
  if (T_local > 0) {
    rc = launch_route(x, L->router, T_local, H, num_experts_global, *rp, s.ids_l, s.w_l, nullptr, s.part,
                      s.counts_g, nullptr, st);
    if (rc) return rc;
  }
  // 2. dispatch
  rc = ep_allgather(ep, x, s.ids_l, s.w_l, T_local, H, k, s.x_all, s.ids_all, s.w_all, st);
  if (rc) return rc;
  // 3. local pairs -> permutation -> grouped FFN over the local experts
  if (cudaMemsetAsync(s.counts, 0, sizeof(int) * E_l, st) != cudaSuccess) return CCUT_ERR_CUDA;
  rc = launch_k(localize_count_kernel, dim3(grid_for((size_t)T * k, 256 * 4)), dim3(256), 0, st,
                (const int32_t*)s.ids_all, (const float*)s.w_all, T * k, expert_lo, E_l, s.ids_loc, s.w_loc, s.counts);
  if (rc) return rc;
  rc = launch_permute(s.ids_loc, s.w_loc, T, k, E_l, 0, 0.f, s.counts, s.offsets, s.row_token, s.row_weight,
                      s.pair_row, st);
  if (rc) return rc;
  const long per_expert = (long)T * k / num_experts_global;  // rows of a local expert, on average
  const ccut_moe_layer rv = with_policy(routed_view(L), per_expert);
  if (rv.kernel == CCUT_KERNEL_MMA) {
    rc = launch_bf16_to_f16(s.x_all, s.ffn.x16, (size_t)T * H, st);
    if (rc) return rc;
  }
  rc = run_ffn(&rv, per_expert, s.x_all, s.ffn, T, k, s.offsets, s.row_token, s.row_weight, s.ybuf, s.status, st);
  if (rc) return rc;
  // 4. per-token sum of the local rows, then reduce-scatter back to the token owners
  rc = launch_combine(s.ybuf, s.pair_row, T, k, H, 0, -1, s.y_part, CCUT_OUT_F32, st);
  if (rc) return rc;
  rc = ep_reduce_scatter(ep, s.y_part, T_local, H, s.y_loc, st);
  if (rc) return rc;
  if (T_local == 0) return CCUT_OK;
  if (shared && cudaStreamWaitEvent(st, ep->join, 0) != cudaSuccess) return CCUT_ERR_CUDA;
  const size_t n4 = (size_t)T_local * H / 4;
  return launch_k(add_cast_kernel, dim3(grid_for(n4, 256)), dim3(256), 0, st, reinterpret_cast<const float4*>(s.y_loc),
                  shared ? reinterpret_cast<const float4*>(s.y_sh) : nullptr, n4, out, out_dtype);
}

}  // extern "C"
