// Shared device helpers for the vxmoe kernels (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "vxmoe.h"

#define VX_DEVICE __device__ __forceinline__
#define VX_HOST_DEVICE __host__ __device__

namespace vx {

constexpr int kWarp = 32;

// ---------------------------------------------------------------------------
// bf16 as bit patterns.  Round-to-nearest-even, NaN kept quiet.
// ---------------------------------------------------------------------------

VX_DEVICE float bf16_to_f32(uint16_t b) { return __uint_as_float(uint32_t(b) << 16); }

VX_DEVICE uint16_t f32_to_bf16(float f) {
  uint32_t u = __float_as_uint(f);
  if ((u & 0x7FFFFFFFu) > 0x7F800000u) return uint16_t((u >> 16) | 0x0040u);
  u += 0x7FFFu + ((u >> 16) & 1u);
  return uint16_t(u >> 16);
}

// Value of f rounded to bf16, kept as float.
VX_DEVICE float bf16r(float f) { return bf16_to_f32(f32_to_bf16(f)); }

// float32 exp(m) rounded to bf16 as if the float32 exp were correctly
// rounded.  The library expf is within a few ulp; when its result sits close
// to a bf16 rounding boundary the value is recomputed in double precision, so
// the bf16 result is the rounding of the exact float32 exp.
VX_DEVICE float bf16_exp(float m) {
  float e = expf(m);
  uint32_t low = __float_as_uint(e) & 0xFFFFu;
  if (low >= 0x7FF0u && low <= 0x8010u) e = float(exp(double(m)));
  return bf16r(e);
}

// MLX's stable bf16 sigmoid: every step rounded to bf16.
// t = exp(|z|); s = 1/(1+t); sigma = z<0 ? s : 1-s.
VX_DEVICE float sigmoid_bf16(float z) {
  float t = bf16_exp(fabsf(z));
  float den = bf16r(__fadd_rn(1.0f, t));
  float s = bf16r(__fdiv_rn(1.0f, den));
  return z < 0.0f ? s : bf16r(__fsub_rn(1.0f, s));
}

// h = silu(g) * u in bf16 (g, u already bf16 values).
VX_DEVICE float silu_mul_bf16(float g, float u) {
  float sg = sigmoid_bf16(g);
  float silu = bf16r(__fmul_rn(g, sg));
  return bf16r(__fmul_rn(silu, u));
}

// ---------------------------------------------------------------------------
// Q4 nibbles.  For the 16-bit half h of a word, nibble p (0..3) is
// (h >> 4p) & 15.  OR-ing the masked half into the float 2^23 and
// subtracting 2^23 yields q * 16^p exactly (q*16^p < 2^16); the matching
// activation is pre-scaled by 16^-p, so each product equals q*x.
// ---------------------------------------------------------------------------

VX_DEVICE float nib_scaled(uint32_t half, int p) {
  return __uint_as_float((half & (0xFu << (4 * p))) | 0x4B000000u) - 8388608.0f;
}

VX_DEVICE uint32_t nibble(uint32_t w, int i) { return (w >> (4 * i)) & 0xFu; }

// ---------------------------------------------------------------------------
// Warp reductions
// ---------------------------------------------------------------------------

template <int WIDTH>
VX_DEVICE float warp_sum(float v) {
#pragma unroll
  for (int o = WIDTH / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o, WIDTH);
  return v;
}

VX_DEVICE float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xFFFFFFFFu, v, o));
  return v;
}

// ---------------------------------------------------------------------------
// Tensor-pipe and load helpers
// ---------------------------------------------------------------------------

VX_DEVICE void mma16816_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                            uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
VX_DEVICE void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                        uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

VX_DEVICE uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}

// 16-byte read-only load that asks L2 to keep the line (evict-last policy):
// the router's rows - 2 MiB per layer, read by every token - stay resident
// while the expert records stream through L2 with an evict-first policy.
VX_DEVICE uint4 ldg_keep(const void* p) {
  uint64_t pol;
  asm("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0,%1,%2,%3}, [%4], %5;"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p), "l"(pol));
  return v;
}

VX_DEVICE uint4 ldg_nc(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// "B order" of an activation row: inside each block of 8 inputs the 16-bit
// slots hold x0 x4 x1 x5 x2 x6 x3 x7, so one 32-bit word is the bf16x2 pair
// that meets the nibble pairs (0,4) (1,5) (2,6) (3,7) of a packed word in an
// MMA fragment.  Returns the slot of logical column `col`.
// Record index of routed expert e in a tiled pool: its slot when the pool
// holds only some experts (slot_of non-null; an entry outside [0, slots) -
// an expert the caller did not make resident - reads slot 0: undefined
// output, in-bounds reads), else e itself.
VX_DEVICE int64_t routed_record(const int32_t* slot_of, int slots, int e) {
  if (!slot_of) return e;
  const int s = __ldg(slot_of + e);
  return (s >= 0 && s < slots) ? s : 0;
}

VX_DEVICE int b_order_col(int col) {
  const int e = col & 7;
  return (col & ~7) | (e < 4 ? 2 * e : 2 * (e - 4) + 1);
}

// Address of expert e's rows in a bank (int64 offsets: a full bank of 512
// experts spans more than 2^31 bytes).
struct Q4Ptr {
  const uint32_t* w;
  const uint16_t* s;
  const uint16_t* b;
};

// ---------------------------------------------------------------------------
// Programmatic dependent launch.  The block's kernels follow one another on
// one stream; each is launched with programmatic stream serialisation
// (launch_chained), so it may become resident while its predecessor still
// runs.  chain_begin() first waits until the predecessor grid has completed
// and its memory is visible (a no-op when the launch had no programmatic
// edge), then lets the successor launch.  Every chained kernel calls it, or
// chain_wait(), before touching global memory.  The streaming GEMV/GEMM
// kernels call chain_wait(): their successors launch only as their CTAs
// exit, so no waiting CTA takes an SM slot from them.
// ---------------------------------------------------------------------------

VX_DEVICE void chain_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

VX_DEVICE void chain_begin() {
  chain_wait();
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

VX_DEVICE Q4Ptr q4_expert(const vx_q4& bank, int e) {
  const int64_t words = int64_t(bank.out) * (bank.in / 8);
  const int64_t groups = int64_t(bank.out) * (bank.in / bank.group_size);
  return {bank.w + int64_t(e) * words, bank.scales + int64_t(e) * groups,
          bank.biases + int64_t(e) * groups};
}

}  // namespace vx

// Host-side launch check used by every entry point.
int vx_cuda_fail(cudaError_t e);
namespace vx {
// Argument checks of vx_moe_block short of the workspace (vx_abi.cu).
int block_args_status(const uint16_t* x, int T, const vx_moe_weights* W, const uint16_t* y);
}  // namespace vx

#define VX_LAUNCH_CHECK()                                   \
  do {                                                      \
    cudaError_t _e = cudaGetLastError();                    \
    if (_e != cudaSuccess) return vx_cuda_fail(_e);         \
  } while (0)
