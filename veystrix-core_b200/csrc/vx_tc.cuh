// tcgen05 / TMEM helpers of the grouped expert GEMMs (sm_100a inline PTX):
// shared-memory matrix descriptors for K-major 128-byte-swizzled operands,
// the kind::f16 instruction descriptor, MMA issue and commit, TMEM loads,
// and the bf16 dequantisation of one packed word.
#pragma once

#include <stdint.h>

#include "vx_async.cuh"
#include "vx_common.cuh"

namespace vx {

constexpr int kGemmRows = 128;          // M of the MMA: weight rows per tile
constexpr int kAtomBytes = 128 * 128;   // one 128-row x 64-input swizzled atom

// K-major, 128-byte swizzle: start address, LBO (unused for this layout),
// SBO = 1024 bytes between 8-row groups, descriptor version 1.  The atom's
// base must be 1024-byte aligned; a K step of 16 inputs adds 32 bytes.
VX_DEVICE uint64_t sw128_desc(uint32_t addr) {
  return uint64_t((addr >> 4) & 0x3FFFu) | (uint64_t(1) << 16) | (uint64_t(1024 >> 4) << 32) |
         (uint64_t(1) << 46) | (uint64_t(2) << 61);
}

// kind::f16: fp32 accumulator, bf16 A and B, both K-major, N (multiple of
// 16, <= 256), M = 128.
VX_DEVICE uint32_t mma_idesc(int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (uint32_t(n >> 3) << 17) | (uint32_t(kGemmRows >> 4) << 24);
}

VX_DEVICE void mma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, bool acc) {
  asm volatile(
      "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(int(acc))
      : "memory");
}

// The same MMA with A read from TMEM: 128 lanes = the 128 rows of A, 16 bf16
// of K packed two per 32-bit column (8 columns per K step).
VX_DEVICE void mma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc, bool acc) {
  asm volatile(
      "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(int(acc))
      : "memory");
}

// 32 consecutive 32-bit columns of this thread's TMEM lane (warp-collective);
// tmem_wait_st waits for this warp's stores.
VX_DEVICE void tmem_st32(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
      "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]),
      "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]),
      "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}
VX_DEVICE void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Arrives on `bar` once every tcgen05 operation this thread issued so far has
// completed.
VX_DEVICE void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}

VX_DEVICE void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
VX_DEVICE void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 16 consecutive fp32 columns of this thread's TMEM lane (warp-collective).
VX_DEVICE void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, "
      "[%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

VX_DEVICE void tmem_alloc(uint32_t slot_smem, uint32_t cols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(slot_smem), "r"(cols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
VX_DEVICE void tmem_dealloc(uint32_t taddr, uint32_t cols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols) : "memory");
}

VX_DEVICE void mbar_init_n(uint32_t bar, uint32_t n) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(n) : "memory");
}
VX_DEVICE void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

VX_DEVICE uint32_t bf16x2_fma(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}

// 8 nibbles of one word -> 8 bf16 weights in B order, w = bf16(s*q + b):
// lop3 gives the exact pair 128+q, the first bf16x2 FMA subtracts 128
// exactly, the second rounds s*q + b once.
VX_DEVICE uint4 dequant_word(uint32_t w, uint32_t s2, uint32_t b2) {
  const uint32_t one = 0x3F803F80u, m128 = 0xC300C300u;
  uint4 o;
  o.x = bf16x2_fma(bf16x2_fma(nib_pair128(w), one, m128), s2, b2);
  o.y = bf16x2_fma(bf16x2_fma(nib_pair128(w >> 4), one, m128), s2, b2);
  o.z = bf16x2_fma(bf16x2_fma(nib_pair128(w >> 8), one, m128), s2, b2);
  o.w = bf16x2_fma(bf16x2_fma(nib_pair128(w >> 12), one, m128), s2, b2);
  return o;
}

VX_DEVICE void sts128(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

}  // namespace vx
