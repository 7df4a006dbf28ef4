// tl_tc_ptx.cuh -- PTX wrappers shared by the tcgen05 kernels (sm_100a):
// mbarriers with bounded waits, TMA tile loads (no multicast), tcgen05 MMA /
// commit / fences, shared-memory matrix descriptors, and the CTA-pair
// (cta_group::2) signalling over cluster addresses.
#pragma once
#include <cuda.h>
#include <cstdint>

namespace tl {
namespace tc {

constexpr long long WAIT_LIMIT_CYCLES = 4000000000LL;  // ~2 s at 1.9 GHz

// --------------------------------------------------------------- PTX helpers
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("{ .reg .b64 st; mbarrier.arrive.shared::cta.b64 st, [%0]; }" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("{ .reg .b64 st; mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1; }" ::"r"(bar), "r"(bytes)
               : "memory");
}
// Waiting threads are suspended by the barrier (up to SUSPEND_NS per try, or
// until the phase completes) instead of spinning: a spinning wait loop issues
// an instruction stream of its own that competes with the working warps for
// issue slots and power.
constexpr uint32_t SUSPEND_NS = 10000000u;
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3; selp.u32 %0, 1, 0, p; }"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(SUSPEND_NS)
      : "memory");
  return ok != 0;
}
// Bounded wait.  Returns false (and raises the abort flag) on expiry or when
// another thread of the CTA has already aborted.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int *abort_flag,
                                          int *err, int code) {
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (*abort_flag) return false;
    if (clock64() - t0 > WAIT_LIMIT_CYCLES) {
      *abort_flag = 1;
      atomicExch(err, code);
      return false;
    }
  }
  return true;
}
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap *map, uint32_t bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{ .reg .pred p; setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p; }" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void tc_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

// Shared-memory matrix descriptor (sm_100 layout: version 1 at bits 46-47,
// layout type at bits 61-63).  Two layouts are used:
//  K-major operands:  128-byte swizzle (type 2), 16-byte chunks XOR row%8;
//                     8-row groups 1 KB apart (SBO), LBO unused.
//  MN-major operands: 128-byte swizzle on a 32-byte base (type 1), 32-byte
//                     chunks XOR row%4 -- the only MN-major layout tcgen05
//                     accepts for tf32; 4-row K groups 512 B apart (SBO),
//                     32-element MN chunks 4 KB apart (LBO).
constexpr uint32_t LAYOUT_SW128 = 2, LAYOUT_SW128_BASE32B = 1;
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo_bytes, uint32_t sbo_bytes,
                                              uint32_t layout) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)layout << 61;
  return d;
}

// The value the tf32 MMA reads from an fp32 word: the low 13 mantissa bits
// are ignored (measured on B200: 1 + 3*2^-12 multiplies as 1.0), so the raw
// tile serves as hi and only lo = x - trunc_tf32(x), exact in fp32, is stored.
__device__ __forceinline__ float tf32_trunc(float x) { return __uint_as_float(__float_as_uint(x) & 0xffffe000u); }

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_map(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
// Arrive on a barrier of either CTA of the pair (default .release.cta
// semantics).  Callers have already ordered their shared-memory writes for the
// tensor pipe with fence.proxy.async.  A .release.cluster arrive here costs
// ~1 us per call (measured: the pair kernel ran at 173 TFLOP/s with it and at
// 246 without).
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait_cl(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{ .reg .pred p; mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3; selp.u32 %0, 1, 0, p; }"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(SUSPEND_NS)
      : "memory");
  return ok != 0;
}
// Non-blocking test of a phase (cluster scope), for polls between work items.
__device__ __forceinline__ bool mbar_test_cl(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{ .reg .pred p; mbarrier.test_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// Cluster-wide barrier of all threads of both CTAs (the non-aligned form:
// lanes of a warp may arrive from different branches).
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}
// Abort raised in this CTA is also written into the peer's flag, so that the
// peer stops waiting for signals that will not come.
__device__ __forceinline__ void pair_abort(volatile int *flag, uint32_t peer_flag, int *err, int code) {
  *flag = 1;
  asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(peer_flag), "r"(1) : "memory");
  atomicExch(err, code);
}
__device__ __forceinline__ bool mbar_wait_pair(uint32_t bar, uint32_t parity, volatile int *flag, uint32_t peer_flag,
                                               int *err, int code) {
  const long long t0 = clock64();
  while (!mbar_try_wait_cl(bar, parity)) {
    if (*flag) return false;
    if (clock64() - t0 > WAIT_LIMIT_CYCLES) {
      pair_abort(flag, peer_flag, err, code);
      return false;
    }
  }
  return true;
}
__device__ __forceinline__ void tc_mma_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{ .reg .pred p; setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::tf32 [%0], %1, %2, %3, p; }" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void tc_mma_pair_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                                uint32_t accumulate) {
  asm volatile(
      "{ .reg .pred p; setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p; }" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive (once the pair's MMAs issued so far have completed) on the barrier at
// this shared-memory offset in both CTAs of the pair.
__device__ __forceinline__ void tc_commit_pair(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::
                   "r"(bar), "h"((uint16_t)0x3)
               : "memory");
}

}  // namespace tc
}  // namespace tl
