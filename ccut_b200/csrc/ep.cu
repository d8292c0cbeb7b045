// ep.cu -- expert-parallel MoE forward, one process per GPU, over NCCL: only routed rows
// cross the links.
//
// Rank r of P holds the routed experts [lo_r, hi_r) (contiguous blocks whose sizes differ by
// at most one, ep_range) plus every shared expert, and its own T_r tokens (T_r may differ
// between ranks; every rank sized its workspace for the same T_cap >= T_r).  One forward:
//   1. route the local tokens against the global router (ids are global expert indices);
//   2. plan (ep_plan_kernel, one CTA per destination d): the local tokens with at least one
//      expert on d, in token order; each gets ONE row in d's segment of the send buffers (its
//      k ids made local to d with -1 for other ranks' experts, its k routing weights, its
//      token), and send_pos[t, d] keeps the row's place for the way back; then
//      ep_gather_kernel (a full grid) copies the bf16 token rows into those places;
//   3. dispatch: grouped ncclSend / ncclRecv of each destination's segment, T_cap rows (the rows
//      past the segment's count carry ids -1 and take no expert), received at s * T_cap for
//      source s.  The segments have a size the host knows, so no count travels to the host and
//      the step never waits on it (the unused tail of a segment crosses the link as well: at
//      small rank counts nearly every token goes to every rank, at 8 ranks about 2/3 of them);
//   5. the received rows through this rank's experts: permute by local expert (a -1 id takes
//      no row), grouped FFN, per-row weighted sum over the row's k slots in slot order (fp32);
//   6. return: each source's segment of partial rows sent back to it as bf16 (one rounding of
//      each partial sum, as the layer's bf16 output has), in its send order;
//   7. out[t] = sum over destinations d = 0..P-1 of the partial row of (t, d), in that fixed
//      order, plus the shared experts, which run data-parallel on the local tokens on a second
//      stream meanwhile.
// The volume per rank is the routed rows only: a token crosses to each rank that owns one of
// its experts once, whatever P is.  The reference runs the experts of one layer in a single
// process (ccut/models/generic.py:364-385, ccut/experts/pipeline.py:123-190); the partitioning
// is new.  One blocking NCCL communicator per handle carries the exchanges.
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
  cudaStream_t side;  // shared experts run here, beside the exchange
  cudaEvent_t fork, join;
};

namespace ccut {
namespace {

constexpr int kPlanThreads = 1024;
constexpr int kMaxWorld = 64;

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

// First routed expert of rank d (contiguous blocks, sizes differing by at most one; the same
// split as ccut_b200.ep.expert_range).
__host__ __device__ inline int ep_lo(int E, int world, int d) {
  const int base = E / world, extra = E % world;
  return d * base + (d < extra ? d : extra);
}

// One CTA per destination rank d: the local tokens with an expert on d, in token order
// (block-wide scan of the flags, 1024 tokens per round), each given a row of d's segment of
// the send buffers; send_pos[t * world + d] = the row's index in the send buffers, or -1, and
// send_tok[row] = t.
__global__ void __launch_bounds__(kPlanThreads) ep_plan_kernel(const int32_t* __restrict__ ids,
                                                               const float* __restrict__ w, int T, int k, int E,
                                                               int world, int seg, int* __restrict__ send_cnt,
                                                               int32_t* __restrict__ send_pos,
                                                               int32_t* __restrict__ send_tok,
                                                               int32_t* __restrict__ ids_send,
                                                               float* __restrict__ w_send) {
  pdl_wait();
  pdl_trigger();
  __shared__ int wsum[kPlanThreads / 32];
  __shared__ int s_total;
  const int d = blockIdx.x, tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int lo = ep_lo(E, world, d), hi = ep_lo(E, world, d + 1);
  int carry = 0;
  for (int base = 0; base < T; base += kPlanThreads) {
    const int t = base + tid;
    bool flag = false;
    if (t < T)
      for (int j = 0; j < k; ++j) {
        const int e = ids[(size_t)t * k + j];
        flag |= e >= lo && e < hi;
      }
    const unsigned bal = __ballot_sync(0xffffffffu, flag);
    if (lane == 0) wsum[wid] = __popc(bal);
    __syncthreads();
    if (wid == 0) {  // exclusive scan of the 32 warp counts
      const int c = wsum[lane];
      int inc = c;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int u = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += u;
      }
      wsum[lane] = inc - c;
      if (lane == 31) s_total = inc;
    }
    __syncthreads();
    const int pos = wsum[wid] + __popc(bal & ((1u << lane) - 1u));
    if (flag) {
      const int row = d * seg + carry + pos;
      send_tok[row] = t;
      send_pos[(size_t)t * world + d] = row;
      for (int j = 0; j < k; ++j) {
        const int e = ids[(size_t)t * k + j];
        ids_send[(size_t)row * k + j] = (e >= lo && e < hi) ? e - lo : -1;
        w_send[(size_t)row * k + j] = w[(size_t)t * k + j];
      }
    } else if (t < T) {
      send_pos[(size_t)t * world + d] = -1;
    }
    carry += s_total;
    __syncthreads();
  }
  // the segment's rows past its count take no expert on the receiving rank
  for (int row = carry + tid; row < seg; row += kPlanThreads)
    for (int j = 0; j < k; ++j) {
      ids_send[((size_t)d * seg + row) * k + j] = -1;
      w_send[((size_t)d * seg + row) * k + j] = 0.f;
    }
  if (tid == 0) send_cnt[d] = carry;
}

// x_send[row] = x[send_tok[row]] for the first send_cnt[d] rows of every destination's segment
// (seg rows each), 16 bytes per thread, grid-stride.
__global__ void __launch_bounds__(256) ep_gather_kernel(const uint16_t* __restrict__ x,
                                                        const int32_t* __restrict__ send_tok,
                                                        const int* __restrict__ send_cnt, int world, int seg, int H,
                                                        uint16_t* __restrict__ x_send) {
  pdl_wait();
  pdl_trigger();
  const int per_row = H / 8;
  const size_t total = (size_t)world * seg * per_row;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int row = static_cast<int>(i / per_row), c = static_cast<int>(i % per_row);
    if (row % seg >= send_cnt[row / seg]) continue;
    reinterpret_cast<uint4*>(x_send + (size_t)row * H)[c] =
        reinterpret_cast<const uint4*>(x + (size_t)send_tok[row] * H)[c];
  }
}

// out[t] = sum_{d = 0..world-1} back[send_pos[t, d]] (bf16 rows that were sent) + shared[t],
// in that order in fp32 -> bf16 or fp32.  One CTA per (token, 1024-column chunk).
__global__ void __launch_bounds__(256) ep_sum_kernel(const uint16_t* __restrict__ back, const int32_t* __restrict__ send_pos,
                                                     const float* __restrict__ shared, int world, int H, void* out,
                                                     int out_dtype) {
  pdl_wait();
  pdl_trigger();
  __shared__ int rows[kMaxWorld];
  const int t = blockIdx.x;
  if (threadIdx.x < world) rows[threadIdx.x] = send_pos[(size_t)t * world + threadIdx.x];
  __syncthreads();
  const int h4n = H / 4, h4 = blockIdx.y * 256 + threadIdx.x;
  if (h4 >= h4n) return;
  const uint2* b4 = reinterpret_cast<const uint2*>(back);
  float4 s = shared ? reinterpret_cast<const float4*>(shared)[(size_t)t * h4n + h4] : make_float4(0.f, 0.f, 0.f, 0.f);
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int d = 0; d < world; ++d) {
    const int r = rows[d];
    if (r >= 0) {
      const uint2 v = b4[(size_t)r * h4n + h4];
      acc.x += __uint_as_float(v.x << 16);
      acc.y += __uint_as_float(v.x & 0xffff0000u);
      acc.z += __uint_as_float(v.y << 16);
      acc.w += __uint_as_float(v.y & 0xffff0000u);
    }
  }
  acc.x += s.x;
  acc.y += s.y;
  acc.z += s.z;
  acc.w += s.w;
  if (out_dtype == CCUT_OUT_BF16) {
    __nv_bfloat162 lo = __floats2bfloat162_rn(acc.x, acc.y), hi = __floats2bfloat162_rn(acc.z, acc.w);
    uint2 pk;
    pk.x = *reinterpret_cast<uint32_t*>(&lo);
    pk.y = *reinterpret_cast<uint32_t*>(&hi);
    reinterpret_cast<uint2*>(static_cast<uint16_t*>(out) + (size_t)t * H)[h4] = pk;
  } else {
    reinterpret_cast<float4*>(static_cast<float*>(out) + (size_t)t * H)[h4] = acc;
  }
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

// The exchange's own scratch (the plan of the last dispatch, kept for its combine).
struct ExScratch {
  int* status;
  int* cnt;          // [world]: rows sent to each destination
  int32_t* send_pos;  // [T_cap, world]
  int32_t* send_tok;  // [world * T_cap] local token of each send row
  uint16_t* x_send;   // [world * T_cap, H]
  int32_t* ids_send;  // [world * T_cap, k]
  float* w_send;      // [world * T_cap, k]
  uint16_t* back;     // [world * T_cap, H] bf16 partial outputs returned to this rank
};

ExScratch carve_ex(Carver& c, int world, int T_cap, int H, int k) {
  ExScratch s{};
  const size_t rows = (size_t)world * T_cap;
  s.status = c.take<int>(64);
  s.cnt = c.take<int>((size_t)world);
  s.send_pos = c.take<int32_t>((size_t)T_cap * world);
  s.send_tok = c.take<int32_t>(rows);
  s.x_send = c.take<uint16_t>(rows * H);
  s.ids_send = c.take<int32_t>(rows * k);
  s.w_send = c.take<float>(rows * k);
  s.back = c.take<uint16_t>(rows * H);
  return s;
}

struct EpScratch {
  ExScratch ex;
  int* sched;     // GEMM work counters of the routed FFN
  int* sh_sched;  // and of the shared-expert FFN (runs concurrently on the side stream)
  float* part;
  int* counts_g;
  int32_t* ids_l;
  float* w_l;
  uint16_t* x_recv;
  int32_t* ids_recv;
  float* w_recv;
  int* counts;
  int32_t* offsets;
  int32_t* row_token;
  float* row_weight;
  int32_t* pair_row;
  FfnScratch ffn;
  float* ybuf;
  uint16_t* y_recv;  // bf16 partial output per received row
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

EpScratch carve_ep(Carver& c, const ccut_moe_layer* L, int E_global, int world, int T_cap, int k) {
  const int H = L->hidden, S = L->num_shared_slices;
  const int R = world * T_cap;  // received rows: every token of every rank at most once
  const ccut_moe_layer rv = routed_view(L);
  EpScratch s{};
  s.ex = carve_ex(c, world, T_cap, H, k);
  s.sched = take_sched(c);
  s.sh_sched = take_sched(c);
  s.part = c.take<float>((size_t)route_scratch_floats_upto(T_cap, E_global, H));
  s.counts_g = c.take<int>(E_global);
  s.ids_l = c.take<int32_t>((size_t)T_cap * k);
  s.w_l = c.take<float>((size_t)T_cap * k);
  s.x_recv = c.take<uint16_t>((size_t)R * H);
  s.ids_recv = c.take<int32_t>((size_t)R * k);
  s.w_recv = c.take<float>((size_t)R * k);
  s.counts = c.take<int>(L->num_experts);
  s.offsets = c.take<int32_t>(L->num_experts + 1);
  s.row_token = c.take<int32_t>((size_t)R * k);
  s.row_weight = c.take<float>((size_t)R * k);
  s.pair_row = c.take<int32_t>((size_t)R * k);
  s.ffn = carve_ffn(c, &rv, R, k, true, s.sched);
  s.ybuf = c.take<float>((size_t)R * k * H);
  s.y_recv = c.take<uint16_t>((size_t)R * H);
  if (S > 0) {
    const ccut_moe_layer sv = shared_view(L);
    const size_t Rs = (size_t)(S + 1) * T_cap;
    s.sh_ids = c.take<int32_t>(T_cap);
    s.sh_w = c.take<float>(T_cap);
    s.sh_counts = c.take<int>(1);
    s.sh_offsets = c.take<int32_t>(S + 2);
    s.sh_row_token = c.take<int32_t>(Rs);
    s.sh_row_weight = c.take<float>(Rs);
    s.sh_pair_row = c.take<int32_t>(T_cap);
    s.sh_ffn = carve_ffn(c, &sv, T_cap, 1, true, s.sh_sched);
    s.sh_ybuf = c.take<float>(Rs * H);
    s.y_sh = c.take<float>((size_t)T_cap * H);
  }
  return s;
}

int check_ep(const ccut_ep* ep) {
  if (!ep || ep->world < 1 || ep->world > kMaxWorld || ep->rank < 0 || ep->rank >= ep->world) return CCUT_ERR_INVALID;
  if (!ep->comm) return CCUT_ERR_NCCL;
  return CCUT_OK;
}

// Steps 2-3: plan and row exchange.  The received rows land in segments of T_cap rows per
// source rank (x_recv, ids_recv, w_recv: world * T_cap rows).  ids are global expert ids
// [T_l, k].
int ep_dispatch(ccut_ep* ep, const uint16_t* x, const int32_t* ids, const float* w, int T_l, int T_cap, int H, int k,
                int E, const ExScratch& s, uint16_t* x_recv, int32_t* ids_recv, float* w_recv, cudaStream_t st) {
  const int P = ep->world;
  int rc = launch_k(ep_plan_kernel, dim3(P), dim3(kPlanThreads), 0, st, ids, w, T_l, k, E, P, T_cap, s.cnt,
                    s.send_pos, s.send_tok, s.ids_send, s.w_send);
  if (rc) return rc;
  if (T_l > 0) {
    size_t blocks = ((size_t)P * T_cap * (H / 8) + 255) / 256;
    if (blocks > 148 * 8) blocks = 148 * 8;
    rc = launch_k(ep_gather_kernel, dim3(static_cast<unsigned>(blocks < 1 ? 1 : blocks)), dim3(256), 0, st, x,
                  (const int32_t*)s.send_tok, (const int*)s.cnt, P, T_cap, H, s.x_send);
    if (rc) return rc;
  }
  if (T_cap == 0) return CCUT_OK;
  if (ncclGroupStart() != ncclSuccess) return CCUT_ERR_NCCL;
  for (int p = 0; p < P; ++p) {
    const size_t r0 = (size_t)p * T_cap;
    ncclSend(s.x_send + r0 * H, (size_t)T_cap * H * 2, ncclUint8, p, ep->comm, st);
    ncclSend(s.ids_send + r0 * k, (size_t)T_cap * k, ncclInt32, p, ep->comm, st);
    ncclSend(s.w_send + r0 * k, (size_t)T_cap * k, ncclFloat32, p, ep->comm, st);
    ncclRecv(x_recv + r0 * H, (size_t)T_cap * H * 2, ncclUint8, p, ep->comm, st);
    ncclRecv(ids_recv + r0 * k, (size_t)T_cap * k, ncclInt32, p, ep->comm, st);
    ncclRecv(w_recv + r0 * k, (size_t)T_cap * k, ncclFloat32, p, ep->comm, st);
  }
  return nccl_settle(ep->comm, ncclGroupEnd(), ep->timeout_s);
}

// Step 6: the partial rows y_recv [world * T_cap, H] (bf16) back to their sources, into s.back.
int ep_return(ccut_ep* ep, const uint16_t* y_recv, int T_cap, int H, const ExScratch& s, cudaStream_t st) {
  const int P = ep->world;
  if (T_cap == 0) return CCUT_OK;
  if (ncclGroupStart() != ncclSuccess) return CCUT_ERR_NCCL;
  for (int p = 0; p < P; ++p) {
    const size_t r0 = (size_t)p * T_cap;
    ncclSend(y_recv + r0 * H, (size_t)T_cap * H, ncclBfloat16, p, ep->comm, st);
    ncclRecv(s.back + r0 * H, (size_t)T_cap * H, ncclBfloat16, p, ep->comm, st);
  }
  return nccl_settle(ep->comm, ncclGroupEnd(), ep->timeout_s);
}

int launch_ep_sum(const ExScratch& s, const float* shared, int T_l, int world, int H, void* out, int out_dtype,
                  cudaStream_t st) {
  if (T_l == 0) return CCUT_OK;
  const dim3 grid(T_l, (H / 4 + 255) / 256);
  return launch_k(ep_sum_kernel, grid, dim3(256), 0, st, (const uint16_t*)s.back, (const int32_t*)s.send_pos, shared,
                  world, H, out, out_dtype);
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
  if (!unique_id || !out || world < 1 || world > kMaxWorld || rank < 0 || rank >= world || !(timeout_s > 0))
    return CCUT_ERR_INVALID;
  *out = nullptr;
  ncclUniqueId id;
  std::memcpy(&id, unique_id, sizeof(id));
  // A blocking communicator: init returns once every rank has joined (the caller bounds
  // that wait: the unique id reaches the ranks through a collective with a timeout, and the
  // process has its own limit); exchanges are enqueued without host polling.
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

size_t ccut_moe_ep_exchange_workspace_bytes(int world, int T_cap, int H, int k) {
  if (world < 1 || world > kMaxWorld || T_cap < 0 || H <= 0 || H % 8 || k < 1 || k > kMaxTopK) return 0;
  Carver c(nullptr);
  carve_ex(c, world, T_cap, H, k);
  return c.off;
}

int ccut_moe_ep_dispatch(ccut_ep* ep, const uint16_t* x, const int32_t* ids, const float* weights, int T_local,
                         int T_cap, int H, int k, int num_experts_global, uint16_t* x_recv, int32_t* ids_recv,
                         float* w_recv, int recv_capacity, int* recv_rows, void* workspace, size_t ws_bytes,
                         ccut_stream_t stream) {
  int rc = check_ep(ep);
  if (rc) return rc;
  PdlScope pdl_scope((long)T_local * ep->world);
  if (T_local < 0 || T_local > T_cap || H <= 0 || H % 8 || k < 1 || k > kMaxTopK || !recv_rows ||
      num_experts_global < ep->world || num_experts_global > kMaxRoutedExperts || recv_capacity < 0)
    return CCUT_ERR_INVALID;
  if ((T_local > 0 && (!x || !ids || !weights)) || (T_cap > 0 && (!x_recv || !ids_recv || !w_recv)) ||
      !workspace)
    return CCUT_ERR_INVALID;
  if ((long)recv_capacity < (long)ep->world * T_cap) return CCUT_ERR_WORKSPACE;
  if (ws_bytes < ccut_moe_ep_exchange_workspace_bytes(ep->world, T_cap, H, k)) return CCUT_ERR_WORKSPACE;
  Carver c(workspace);
  const ExScratch s = carve_ex(c, ep->world, T_cap, H, k);
  rc = ep_dispatch(ep, x, ids, weights, T_local, T_cap, H, k, num_experts_global, s, x_recv, ids_recv, w_recv,
                   stream);
  if (rc == CCUT_OK) *recv_rows = ep->world * T_cap;
  return rc;
}

int ccut_moe_ep_combine(ccut_ep* ep, const uint16_t* y_recv, int T_local, int T_cap, int H, int k, float* y_local,
                        void* workspace, size_t ws_bytes, ccut_stream_t stream) {
  int rc = check_ep(ep);
  if (rc) return rc;
  PdlScope pdl_scope((long)T_local * ep->world);
  if (T_local < 0 || T_local > T_cap || H <= 0 || H % 8 || k < 1 || k > kMaxTopK) return CCUT_ERR_INVALID;
  if ((T_local > 0 && !y_local) || (T_cap > 0 && !y_recv) || !workspace) return CCUT_ERR_INVALID;
  if (ws_bytes < ccut_moe_ep_exchange_workspace_bytes(ep->world, T_cap, H, k)) return CCUT_ERR_WORKSPACE;
  Carver c(workspace);
  const ExScratch s = carve_ex(c, ep->world, T_cap, H, k);
  rc = ep_return(ep, y_recv, T_cap, H, s, stream);
  if (rc) return rc;
  return launch_ep_sum(s, nullptr, T_local, ep->world, H, y_local, CCUT_OUT_F32, stream);
}

size_t ccut_moe_ep_forward_workspace_bytes(const ccut_moe_layer* L, int num_experts_global, int world, int T_cap,
                                           int top_k) {
  if (check_layer(L) || world < 1 || world > kMaxWorld || T_cap < 0 || top_k < 1 || top_k > kMaxTopK ||
      num_experts_global < L->num_experts)
    return 0;
  Carver c(nullptr);
  carve_ep(c, L, num_experts_global, world, T_cap, top_k);
  return c.off;
}

int ccut_moe_ep_forward(ccut_ep* ep, const ccut_moe_layer* L, int expert_lo, int num_experts_global,
                        const ccut_route_params* rp, const uint16_t* x, int T_local, int T_cap, void* out,
                        int out_dtype, void* workspace, size_t ws_bytes, ccut_stream_t stream) {
  int rc = check_ep(ep);
  if (rc) return rc;
  PdlScope pdl_scope((long)T_local * ep->world);  // PDL for decode-sized calls
  rc = check_layer(L);
  if (rc) return rc;
  if (!L->router) return CCUT_ERR_INVALID;
  if (num_experts_global < ep->world || num_experts_global > kMaxRoutedExperts ||
      expert_lo != ep_lo(num_experts_global, ep->world, ep->rank) ||
      expert_lo + L->num_experts != ep_lo(num_experts_global, ep->world, ep->rank + 1))
    return CCUT_ERR_INVALID;  // the layer must hold exactly this rank's block of experts
  rc = check_route(rp, num_experts_global);
  if (rc) return rc;
  if (out_dtype != CCUT_OUT_BF16 && out_dtype != CCUT_OUT_F32) return CCUT_ERR_INVALID;
  if (T_local < 0 || T_local > T_cap) return CCUT_ERR_INVALID;
  // every rank must take part in the exchanges, so an empty local batch still runs them
  const int k = rp->top_k, H = L->hidden, E_l = L->num_experts, S = L->num_shared_slices;
  if (T_local > 0 && (!x || !out)) return CCUT_ERR_INVALID;
  if (!workspace) return CCUT_ERR_INVALID;
  if (ws_bytes < ccut_moe_ep_forward_workspace_bytes(L, num_experts_global, ep->world, T_cap, k))
    return CCUT_ERR_WORKSPACE;
  cudaStream_t st = stream;
  Carver c(workspace);
  EpScratch s = carve_ep(c, L, num_experts_global, ep->world, T_cap, k);
  int* status = s.ex.status;

  // 7 (forked). shared experts on the local tokens, on the side stream: no routed pair is
  //    valid there, so every row belongs to a shared slice (rows s * T_local + t)
  const bool shared = S > 0 && T_local > 0;
  if (shared) {
    cudaStream_t ss = ep->side;
    if (cudaEventRecord(ep->fork, st) != cudaSuccess || cudaStreamWaitEvent(ss, ep->fork, 0) != cudaSuccess)
      return CCUT_ERR_CUDA;
    if (cudaMemsetAsync(s.sh_ids, 0xFF, sizeof(int32_t) * T_local, ss) != cudaSuccess) return CCUT_ERR_CUDA;
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
                 0, status, ss);
    if (rc) return rc;
    rc = launch_combine(s.sh_ybuf, 0, s.sh_pair_row, T_local, 1, H, S, 0, s.y_sh, CCUT_OUT_F32, ss);
    if (rc) return rc;
    if (cudaEventRecord(ep->join, ss) != cudaSuccess) return CCUT_ERR_CUDA;
  }
  // 1. route the local tokens (global expert ids)
  if (T_local > 0) {
    rc = launch_route(x, L->router, T_local, H, num_experts_global, *rp, s.ids_l, s.w_l, nullptr, s.part,
                      s.counts_g, nullptr, st);
    if (rc) return rc;
  }
  // 2-3. plan, routed rows
  const int R = ep->world * T_cap;
  rc = ep_dispatch(ep, x, s.ids_l, s.w_l, T_local, T_cap, H, k, num_experts_global, s.ex, s.x_recv, s.ids_recv,
                   s.w_recv, st);
  if (rc) return rc;
  // 5. received rows -> permutation -> grouped FFN over the local experts -> per-row sums
  if (R > 0) {
    rc = launch_count(s.ids_recv, R * k, E_l, s.counts, st);
    if (rc) return rc;
    rc = launch_permute(s.ids_recv, s.w_recv, R, k, E_l, 0, 0.f, s.counts, s.offsets, s.row_token, s.row_weight,
                        s.pair_row, st);
    if (rc) return rc;
    // rows of a local expert, on average, when the ranks carry T_cap tokens each
    const long per_expert = (long)T_cap * ep->world * k / num_experts_global;
    const ccut_moe_layer rv = with_policy(routed_view(L), per_expert);
    if (rv.kernel == CCUT_KERNEL_MMA) {
      rc = launch_bf16_to_f16(s.x_recv, s.ffn.x16, (size_t)R * H, st);
      if (rc) return rc;
    }
    // the partial rows return in bf16, so the weighted rows are bf16 too
    rc = run_ffn(&rv, per_expert, s.x_recv, s.ffn, R, k, s.offsets, s.row_token, s.row_weight, s.ybuf, 1, status, st);
    if (rc) return rc;
    rc = launch_combine(s.ybuf, 1, s.pair_row, R, k, H, 0, -1, s.y_recv, CCUT_OUT_BF16, st);
    if (rc) return rc;
  }
  // 6. partial rows back to their owners
  rc = ep_return(ep, s.y_recv, T_cap, H, s.ex, st);
  if (rc) return rc;
  if (T_local == 0) return CCUT_OK;
  if (shared && cudaStreamWaitEvent(st, ep->join, 0) != cudaSuccess) return CCUT_ERR_CUDA;
  // 7. out[t] = partials in destination order + shared experts
  return launch_ep_sum(s.ex, shared ? s.y_sh : nullptr, T_local, ep->world, H, out, out_dtype, st);
}

}  // extern "C"
