// permute_static.cu -- ccut_moe_permute_static: the token permutation with its scratch in
// a fixed device array of this library instead of a caller workspace.
//
// Who needs it: a host that has no device allocator to hand (a plain C, cgo or ctypes
// caller that never linked a CUDA memory pool) or one whose device memory plan is fixed at
// start-up and forbids any allocation once steps run.  Such a caller cannot size and pass
// the per-expert counter workspace of ccut_moe_permute; this entry point needs only the
// caller's input and output buffers.  It allocates nothing: no cudaMalloc / cudaFree, no
// allocating library routine.
//
// Scratch: kStaticCounters int32 counters (one per routed expert), zeroed on the stream by
// every call before the counting kernel runs.  Nothing the caller passes must start at
// zero: the permutation kernel writes every pair_row entry itself (-1 for a pair without an
// expert), exactly as in ccut_moe_permute.  Like ccut_moe_permute, a call of at most 256
// tokens launches its kernels with programmatic dependent launch.
//
// Setup: the first call on each device (with that device current) resolves the device
// address of the array once with cudaGetSymbolAddress and caches it.  Make that first call
// before any stream capture begins.  The array is shared by every call on a device, so
// calls that overlap in time on one device (two streams, two host threads) race on it;
// serialise them.
#include <atomic>
#include <mutex>

#include "kernels.cuh"

namespace ccut {
namespace {

constexpr int kStaticCounters = CCUT_PERMUTE_STATIC_MAX_EXPERTS;
constexpr int kMaxDevices = 64;
constexpr int kMaxTopKStatic = 16;

// Per-expert counters of the permutation; 1 KiB per device.
static __device__ __align__(256) int g_permute_counts[kStaticCounters];

std::mutex g_setup_mutex;
std::atomic<int*> g_counts_ptr[kMaxDevices];

// Device address of g_permute_counts on the current device (nullptr on failure).  After the
// first call on a device this is one atomic load; the lock only guards the lookup itself.
int* static_counts() {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  int* cached = g_counts_ptr[dev].load(std::memory_order_acquire);
  if (cached) return cached;
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  cached = g_counts_ptr[dev].load(std::memory_order_relaxed);
  if (!cached) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_permute_counts) != cudaSuccess || !p) return nullptr;
    cached = static_cast<int*>(p);
    g_counts_ptr[dev].store(cached, std::memory_order_release);
  }
  return cached;
}

}  // namespace
}  // namespace ccut

using namespace ccut;

extern "C" int ccut_moe_permute_static(const int32_t* ids, const float* weights, int T, int k, int E,
                                       int num_shared_slices, float shared_gate, int32_t* offsets,
                                       int32_t* row_token, float* row_weight, int32_t* pair_row,
                                       ccut_stream_t stream) {
  if (E > kStaticCounters) return CCUT_ERR_UNSUPPORTED;  // beyond the fixed scratch
  if (T < 0 || k < 1 || k > kMaxTopKStatic || E < 1 || num_shared_slices < 0 ||
      E + num_shared_slices > kMaxExperts)
    return CCUT_ERR_INVALID;
  if (!offsets || !row_token || !row_weight || !pair_row || (T > 0 && (!ids || !weights))) return CCUT_ERR_INVALID;
  int* counts = static_counts();
  if (!counts) return CCUT_ERR_CUDA;
  PdlScope pdl_scope(T);  // PDL for decode-sized calls, as in ccut_moe_permute
  int rc = launch_count(ids, T * k, E, counts, stream);  // zeroes counts[0, E) first
  if (rc) return rc;
  return launch_permute(ids, weights, T, k, E, num_shared_slices, shared_gate, counts, offsets, row_token,
                        row_weight, pair_row, stream);
}
