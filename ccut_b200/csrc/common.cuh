// common.cuh -- sm_100a device helpers shared by the MoE kernels.
//
// Inline-PTX wrappers for mbarriers, bulk (non-tensor) async copies, ldmatrix, the
// m16n8k16 tensor-core MMA and the e4m3 -> f16 convert.  Every spin on an mbarrier is
// bounded by a clock budget: when it runs out the waiter records CCUT_ERR_TIMEOUT in
// the workspace status word and the kernel unwinds instead of hanging the GPU.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/ccut_moe.h"

#define CCUT_DEVICE __device__ __forceinline__

namespace ccut {

// About one second at the B200's 1.965 GHz boost clock.
constexpr long long kWaitBudgetCycles = 2000000000LL;

CCUT_DEVICE uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- error word --------------------------------------------------------------------
CCUT_DEVICE void record_error(int* status, int code) {
  if (status) atomicCAS(status, 0, code);
}

// ---- mbarrier ----------------------------------------------------------------------
CCUT_DEVICE void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

CCUT_DEVICE void mbar_arrive(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.release.cta.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
      : "memory");
}

CCUT_DEVICE void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(smem_u32(bar)),
      "r"(bytes)
      : "memory");
}

CCUT_DEVICE bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait for the phase with `parity` to complete.  Returns false on timeout (the
// status word then holds CCUT_ERR_TIMEOUT).  `budget` in SM clock cycles.
CCUT_DEVICE bool mbar_wait(uint64_t* bar, uint32_t parity, int* status, long long budget = kWaitBudgetCycles) {
  if (mbar_try_wait(bar, parity)) return true;
  long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > budget) {
      record_error(status, CCUT_ERR_TIMEOUT);
      return false;
    }
  }
  return true;
}

CCUT_DEVICE bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded busy wait (non-suspending test_wait) for single-thread roles whose wake-up
// latency is on the critical path (MMA issue, TMA producer).
CCUT_DEVICE bool mbar_spin(uint64_t* bar, uint32_t parity, int* status, long long budget = kWaitBudgetCycles) {
  if (mbar_test_wait(bar, parity)) return true;
  long long t0 = clock64();
  while (!mbar_test_wait(bar, parity)) {
    if (clock64() - t0 > budget) {
      record_error(status, CCUT_ERR_TIMEOUT);
      return false;
    }
  }
  return true;
}

// ---- bulk async copy global -> shared (no tensor map, one destination CTA) ---------
// dst and src 16-byte aligned, bytes a multiple of 16.
CCUT_DEVICE void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// ---- cp.async (16 bytes per thread; src-size 0 writes zeros) ---------------------------
CCUT_DEVICE void cp_async16(void* dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(valid ? 16 : 0)
               : "memory");
}
CCUT_DEVICE void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
CCUT_DEVICE void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// ---- ldmatrix / mma ------------------------------------------------------------------
CCUT_DEVICE void ldmatrix_x4(uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3, const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(smem_u32(p)));
}

CCUT_DEVICE void ldmatrix_x2(uint32_t& r0, uint32_t& r1, const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];"
               : "=r"(r0), "=r"(r1)
               : "r"(smem_u32(p)));
}

// D (16x8 f32) += A (16x16) * B (16x8); A/B both bf16 (kBf16 = true) or both f16.
template <bool kBf16>
CCUT_DEVICE void mma_16816(float* d, const uint32_t* a, uint32_t b0, uint32_t b1) {
  if constexpr (kBf16) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
}

// ---- dequant primitives ----------------------------------------------------------------
// AWQ nibbles -> f16x2 without shifting them down: OR-ing the nibbles at bits [0,4) and
// [16,20) into the mantissa of f16 1024.0 (0x6400) gives 1024 + q, the nibbles at bits
// [4,8) and [20,24) give 1024 + 16 q.  Then (1024 + q) - (1024 + z) and
// (1024 + 16 q) * 1/16 - (64 + z) are q - z, exact (one rounding of an exact result).
CCUT_DEVICE uint32_t nib_lo_to_f16x2_minus(uint32_t w, uint32_t z1024) {
  uint32_t v, r;
  asm("lop3.b32 %0, %1, 0x000F000F, 0x64006400, 0xEA;" : "=r"(v) : "r"(w));
  asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(v), "r"(z1024));
  return r;
}
CCUT_DEVICE uint32_t nib_hi_to_f16x2_minus(uint32_t w, uint32_t neg_z64) {
  uint32_t v, r;
  asm("lop3.b32 %0, %1, 0x00F000F0, 0x64006400, 0xEA;" : "=r"(v) : "r"(w));
  asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(v), "r"(0x2C002C00u), "r"(neg_z64));  // 0x2C00 = 1/16
  return r;
}
// f16x2 (1024 + z, 1024 + z) and (-(64 + z), -(64 + z)) for a zero-point z in [0, 16).
CCUT_DEVICE uint32_t zero_pair_f16_1024(uint32_t z) {
  const uint32_t h = 0x6400u | (z & 0xFu);
  return h | (h << 16);
}
CCUT_DEVICE uint32_t zero_pair_f16_neg64(uint32_t z) {
  const uint32_t h = 0xD400u + ((z & 0xFu) << 4);
  return h | (h << 16);
}

// Two e4m3 bytes (low byte = element 0) -> f16x2, exact (NaN codes -> NaN).
CCUT_DEVICE uint32_t e4m3x2_to_f16x2(uint16_t v) {
  uint32_t r;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(r) : "h"(v));
  return r;
}

CCUT_DEVICE float silu(float g) { return g / (1.0f + expf(-g)); }

}  // namespace ccut
