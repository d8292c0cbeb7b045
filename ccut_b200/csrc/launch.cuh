// launch.cuh -- programmatic dependent launch (PDL) for the kernels of the layer path.
//
// A step of the layer is a chain of short kernels (route, permute, the two grouped GEMMs,
// combine) on one stream; at decode sizes the launch latency between them is a sizable
// part of the step.  Each kernel is launched with programmatic stream serialization, so
// that it is scheduled while its predecessor is still running, and starts with
//   pdl_wait()     -- griddepcontrol.wait: returns once the predecessor grid has completed
//                     and its memory is visible; nothing is read or written before it;
//   pdl_trigger()  -- griddepcontrol.launch_dependents: lets the successor's launch begin.
// Both are no-ops for a kernel launched without the attribute (CCUT_PDL=0, or a
// predecessor that is a memset, a copy or another library's kernel, which then orders the
// launch as usual).
//
// Policy (measured on B200): the attribute is set for calls of at most kPdlMaxTokens tokens,
// where it shortened decode steps by 3-14%; above that (prefill) it made the staged layer
// step ~2% slower, so larger calls launch as usual.  Each C entry point opens a PdlScope for
// its call; launches outside any scope are ordinary.
#pragma once

#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <utility>

#include "../../include/ccut_moe.h"

namespace ccut {

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// False when the environment sets CCUT_PDL=0 (measurement); read once.
bool pdl_enabled();

constexpr int kPdlMaxTokens = 256;
extern thread_local bool g_pdl_on;  // launches of this thread use PDL while set
struct PdlScope {
  bool prev;
  explicit PdlScope(long tokens) : prev(g_pdl_on) { g_pdl_on = tokens <= kPdlMaxTokens && pdl_enabled(); }
  ~PdlScope() { g_pdl_on = prev; }
  PdlScope(const PdlScope&) = delete;
  PdlScope& operator=(const PdlScope&) = delete;
};

// Raises the dynamic shared-memory limit of `kern` to `bytes` on the current device, once
// per device (the attribute belongs to the device's context, so a process that drives
// several GPUs sets it on each).  `done` is the caller's per-kernel set of devices (bit d).
template <typename K>
int ensure_smem_limit(K kern, size_t bytes, std::atomic<uint64_t>& done) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return CCUT_ERR_CUDA;
  const uint64_t bit = dev >= 0 && dev < 64 ? (uint64_t)1 << dev : 0;
  if (bit && (done.load(std::memory_order_acquire) & bit)) return CCUT_OK;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes) != cudaSuccess)
    return CCUT_ERR_CUDA;
  done.fetch_or(bit, std::memory_order_release);
  return CCUT_OK;
}

// kern<<<grid, block, smem, st>>>(args...), with programmatic stream serialization inside a
// PdlScope for a small call.
template <typename... KArgs, typename... Args>
int launch_k(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = g_pdl_on ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...) == cudaSuccess ? CCUT_OK : CCUT_ERR_CUDA;
}

}  // namespace ccut
