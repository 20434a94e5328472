// Asynchronous-copy, mbarrier and shared-memory helpers of the GEMV kernels
// (sm_100a inline PTX).  No cluster multicast anywhere: every copy lands in
// the issuing CTA's own shared memory.
#pragma once

#include <stdint.h>

#include "vx_common.cuh"

namespace vx {

// Bounded mbarrier waits: after a second (or this many polls) the waiter
// gives up and the kernel records an error bit instead of waiting forever.
constexpr uint32_t kSpinLimit = 1u << 24;

// {128 + (w & 15), 128 + ((w >> 16) & 15)} as bf16x2 (exact): one lop3 with
// the bf16 pattern of 128.0 (0x4300) in each half.
VX_DEVICE uint32_t nib_pair128(uint32_t w_shifted) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(w_shifted), "r"(0x000F000Fu), "r"(0x43004300u));
  return r;
}

VX_DEVICE uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// cp.async copies.  src_bytes = 0 writes zeros without reading; the _if form
// issues nothing when the predicate is false.
VX_DEVICE void cp16_if(uint32_t dst, const void* src, int src_bytes, bool pred) {
  asm volatile(
      "{ .reg .pred p; setp.ne.b32 p, %3, 0; @p cp.async.cg.shared.global [%0], [%1], 16, %2; }" ::"r"(dst),
      "l"(src), "r"(src_bytes), "r"(int(pred))
      : "memory");
}
VX_DEVICE void cp4(uint32_t dst, const void* src, bool valid) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(dst), "l"(src), "r"(valid ? 4 : 0)
               : "memory");
}
VX_DEVICE void cp8(uint32_t dst, const void* src, bool valid) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(dst), "l"(src), "r"(valid ? 8 : 0)
               : "memory");
}
VX_DEVICE void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
VX_DEVICE void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

VX_DEVICE uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
  return v;
}
// Named CTA barrier `id` (1..15; 0 is __syncthreads') over `count` threads,
// a multiple of 32: arrive signals without waiting (the producer's side,
// release), sync waits until `count` threads have arrived or synced.  The
// non-aligned forms: each thread counts for itself, so a warp that diverged
// just before (a lane-0 branch) still counts 32 and no more.
VX_DEVICE void named_arrive(int id, int count) {
  asm volatile("barrier.arrive %0, %1;" ::"r"(id), "r"(count) : "memory");
}
VX_DEVICE void named_sync(int id, int count) {
  asm volatile("barrier.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

VX_DEVICE uint32_t lds32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}
VX_DEVICE uint2 lds64(uint32_t addr) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
  return v;
}

// mbarriers with an arrival count of 1 (the issuing lane).
VX_DEVICE void mbar_init(uint32_t bar) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar) : "memory");
}
VX_DEVICE void mbar_expect(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
VX_DEVICE bool mbar_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// try_wait with a suspend-time hint: a thread whose phase is not complete
// sleeps in the barrier (woken when the phase completes, or after `ns`)
// instead of polling, so waiting warps leave the issue slots to the warps
// that compute.
VX_DEVICE bool mbar_try_sleep(uint32_t bar, uint32_t parity, uint32_t ns) {
  uint32_t ok;
  asm volatile(
      "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3; selp.u32 %0, 1, 0, p; }"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(ns)
      : "memory");
  return ok != 0;
}
VX_DEVICE uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
constexpr uint32_t kWaitSleepNs = 4000;
constexpr uint64_t kWaitLimitNs = 1000000000ull;   // one second

// Bounded wait for warps that share the SM with computing warps: false when
// a second went by without the phase completing.
VX_DEVICE bool mbar_wait(uint32_t bar, uint32_t parity) {
  if (mbar_try(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t i = 0; i < kSpinLimit; ++i) {
    if (mbar_try_sleep(bar, parity, kWaitSleepNs)) return true;
    if (global_ns() - t0 > kWaitLimitNs) return false;
  }
  return false;
}

// Bounded polling wait for a single-thread role on a pipeline's critical
// path (a producer or an MMA issuer): no sleep, so no wake-up latency; one
// thread polling costs the other warps little issue bandwidth.
VX_DEVICE bool mbar_wait_spin(uint32_t bar, uint32_t parity) {
  if (mbar_try(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t i = 0; i < kSpinLimit; ++i) {
    if (mbar_try(bar, parity)) return true;
    if ((i & 255) == 255 && global_ns() - t0 > kWaitLimitNs) return false;
  }
  return false;
}

// 2-D tiled TMA load (no multicast) completing on an mbarrier.
VX_DEVICE void tma_load_2d(uint32_t dst, const void* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

// Linear bulk copy global -> own shared memory (no multicast), completing on
// an mbarrier.  dst, src 16-byte aligned; bytes a multiple of 16.  The
// evict-first policy keeps streamed weights from displacing reused data in L2.
VX_DEVICE void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], "
      "%4;" ::"r"(dst),
      "l"(src), "r"(bytes), "r"(bar), "l"(policy)
      : "memory");
}

VX_DEVICE uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
VX_DEVICE uint64_t policy_evict_normal() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(p));
  return p;
}
VX_DEVICE uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

}  // namespace vx
