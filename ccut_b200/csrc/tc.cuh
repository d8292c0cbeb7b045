// tc.cuh -- tcgen05 (5th-generation tensor core) helpers for sm_100a.
//
// Tensor-memory allocation, MMA issue with the A operand in tensor memory, commits to
// mbarriers, tensor-memory loads/stores, shared-memory matrix descriptors, and the tiled
// TMA load used to stage the activation operand.  Descriptor bit layouts follow the
// public sm_100 UMMA descriptor definitions (CUTLASS cute/arch/mma_sm100_desc.hpp).
#pragma once

#include "common.cuh"

namespace ccut {
namespace tc {

// ---- tensor memory --------------------------------------------------------------------
// Whole-warp collective: allocate `ncols` (power of two >= 32) columns, address -> *dst.
CCUT_DEVICE void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
CCUT_DEVICE void tmem_relinquish() { asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::); }
CCUT_DEVICE void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

CCUT_DEVICE void fence_before_sync() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
CCUT_DEVICE void fence_after_sync() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
CCUT_DEVICE void wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
CCUT_DEVICE void wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 32 lanes x 32 consecutive 32-bit columns per warp (thread = lane, 32 registers).
CCUT_DEVICE void st_32x32b_x32(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]),
      "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]),
      "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}

CCUT_DEVICE void ld_32x32b_x32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
      "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]),
        "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
        "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr)
      : "memory");
}

CCUT_DEVICE void st_32x32b_x16(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}

CCUT_DEVICE void ld_32x32b_x16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr)
      : "memory");
}

// ---- MMA -------------------------------------------------------------------------------
// Instruction descriptor, kind::f16: A = B = f16, D = f32, both K-major, M = 128.
CCUT_DEVICE uint32_t idesc_f16_m128(uint32_t n) {
  return (1u << 4)            // D format f32
         | (0u << 7)          // A f16
         | (0u << 10)         // B f16
         | ((n >> 3) << 17)   // N / 8
         | ((128u >> 4) << 24);  // M / 16
}

// Shared-memory descriptor of a K-major operand in the 128-byte swizzle layout: rows of
// 128 bytes, 8-row groups 1024 bytes apart.  `saddr` is the shared-space byte address.
CCUT_DEVICE uint64_t sdesc_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)(1) << 16;             // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;     // stride byte offset: 8 rows x 128 B
  d |= (uint64_t)1 << 46;               // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;               // 128-byte swizzle
  return d;
}

// D[tmem] (+)= A[tmem] * B[smem desc]; issued by one thread.
CCUT_DEVICE void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
      : "memory");
}

// mbarrier arrives once when every MMA this thread issued before it has completed.
CCUT_DEVICE void commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// ---- TMA tiled load into this CTA only ------------------------------------------------------
CCUT_DEVICE void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

CCUT_DEVICE void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---- CTA pairs (cta_group::2): one MMA of M = 256 spans the tensor cores of two SMs -------
// A cluster of two CTAs: rank 0 (the "leader") issues the MMAs; each CTA holds its 128 rows
// of A and its half of the N columns of B in its own shared memory at the same offsets, and
// its 128 rows of D in its own tensor memory.

CCUT_DEVICE uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
CCUT_DEVICE void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// shared::cluster address of the object at the same offset as `local` in CTA `rank` of the cluster.
CCUT_DEVICE uint32_t mapa(const void* local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(local)), "r"(rank));
  return r;
}

CCUT_DEVICE void tmem_alloc2(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
CCUT_DEVICE void tmem_relinquish2() { asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::); }
CCUT_DEVICE void tmem_dealloc2(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// Instruction descriptor, kind::f16 with A = B = bf16, D = f32, both K-major, M = 256.
CCUT_DEVICE uint32_t idesc_bf16_m256(uint32_t n) {
  return (1u << 4)            // D format f32
         | (1u << 7)          // A bf16
         | (1u << 10)         // B bf16
         | ((n >> 3) << 17)   // N / 8
         | ((256u >> 4) << 24);  // M / 16
}

// D[tmem] (+)= A[smem desc] * B[smem desc] over the CTA pair; issued by one thread of rank 0.
CCUT_DEVICE void mma_ss2(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive once on the mbarrier at the same offset as `bar` in every CTA of `mask`, when all
// MMAs this thread issued before it have completed.
CCUT_DEVICE void commit2_mc(uint64_t* bar, uint16_t mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(mask)
      : "memory");
}

// Arrive on an mbarrier given by its shared::cluster address (this CTA's or the peer's), with
// the default (CTA-scope) release, as the CUTLASS sm100 pair pipelines signal the peer: a
// cluster-scope release costs the arriving thread ~1.5k clk per call (measured on B200).
// Operand tiles written by threads are handed to the tensor cores by fence_proxy_async_smem
// before the arrival.
CCUT_DEVICE void mbar_arrive_cl(uint32_t cl_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cl_addr) : "memory");
}
CCUT_DEVICE void mbar_arrive_expect_tx_cl(uint32_t cl_addr, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cluster.b64 _, [%0], %1;" ::"r"(cl_addr), "r"(bytes) : "memory");
}
// Wait on a barrier of this CTA that arrivals from the peer CTA complete (cluster-scope
// acquire), bounded like mbar_spin.
CCUT_DEVICE bool mbar_try_wait_cl(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Non-suspending variant for the MMA-issuing thread, whose wake-up latency is on the
// critical path.
CCUT_DEVICE bool mbar_test_wait_cl(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
CCUT_DEVICE bool mbar_spin_cl(uint64_t* bar, uint32_t parity, int* status) {
  if (mbar_test_wait_cl(bar, parity)) return true;
  long long t0 = clock64();
  while (!mbar_test_wait_cl(bar, parity)) {
    if (clock64() - t0 > kWaitBudgetCycles) {
      record_error(status, CCUT_ERR_TIMEOUT);
      return false;
    }
  }
  return true;
}
CCUT_DEVICE bool mbar_wait_cl(uint64_t* bar, uint32_t parity, int* status) {
  if (mbar_try_wait_cl(bar, parity)) return true;
  long long t0 = clock64();
  while (!mbar_try_wait_cl(bar, parity)) {
    if (clock64() - t0 > kWaitBudgetCycles) {
      record_error(status, CCUT_ERR_TIMEOUT);
      return false;
    }
  }
  return true;
}

// TMA tiled load into this CTA's shared memory whose completion is counted on the mbarrier
// at shared::cluster address `bar_cl` (the pair leader's), no multicast.
CCUT_DEVICE void tma_load_2d_pair(void* dst, const CUtensorMap* map, int x, int y, uint32_t bar_cl) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, "
      "%3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar_cl)
      : "memory");
}

// 32-bit store to a shared::cluster address (this CTA's or the peer's shared memory).
CCUT_DEVICE void st_cluster_u32(uint32_t cl_addr, uint32_t v) {
  asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(cl_addr), "r"(v) : "memory");
}
// Arrival that publishes this thread's earlier stores (also to the peer's shared memory) to a
// waiter on either CTA of the cluster (cluster-scope release; a waiter acquires with
// mbar_wait_cl).
CCUT_DEVICE void mbar_arrive_release_cl(uint32_t cl_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cl_addr) : "memory");
}

// Shared-memory writes of this thread become visible to the tensor cores' async proxy.
CCUT_DEVICE void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

template <uint32_t N>
CCUT_DEVICE void setmaxnreg_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}
template <uint32_t N>
CCUT_DEVICE void setmaxnreg_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}

}  // namespace tc
}  // namespace ccut
