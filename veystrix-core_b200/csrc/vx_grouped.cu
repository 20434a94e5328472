// Grouped Q4 affine projection over expert-sorted items (sm_100a).
//
// One tile = one expert x a block of output rows.  The tile stages the x rows
// of its items in shared memory (float32, pre-scaled for the nibble trick of
// vx_common.cuh) and every lane streams its groups of the packed weight rows
// with 128-bit loads: one 16-byte load is exactly one quant group of 32
// inputs, so a lane applies one scale and one bias per load.  Per group the
// lane forms sum(q*x) and uses sum(x) for the bias, as MLX's qmv does
// (models/flashnext/metal_runtime.py:1014-1029), then the partial sums meet
// in a warp-shuffle reduction.  Gate/up mode reads the gate and up rows of
// the same output index and applies the bf16 SwiGLU sequence in the
// epilogue (metal_runtime.py:267-285), writing h in bf16.
#include "vx_common.cuh"
#include "vx_launch.h"

namespace vx {

constexpr int kTN = 4;          // items per staging pass
constexpr int kThreads = 256;

VX_DEVICE float q4_dot_group(const uint4 w, const float4* xv) {
  const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
  float a0 = 0.f, a1 = 0.f;
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const uint32_t lo = ws[c], hi = ws[c] >> 16;
    const float4 xl = xv[2 * c], xh = xv[2 * c + 1];
    a0 = fmaf(nib_scaled(lo, 0), xl.x, a0);
    a1 = fmaf(nib_scaled(lo, 1), xl.y, a1);
    a0 = fmaf(nib_scaled(lo, 2), xl.z, a0);
    a1 = fmaf(nib_scaled(lo, 3), xl.w, a1);
    a0 = fmaf(nib_scaled(hi, 0), xh.x, a0);
    a1 = fmaf(nib_scaled(hi, 1), xh.y, a1);
    a0 = fmaf(nib_scaled(hi, 2), xh.z, a0);
    a1 = fmaf(nib_scaled(hi, 3), xh.w, a1);
  }
  return a0 + a1;
}

template <int LPR, int NR, bool GATEUP>
__global__ void __launch_bounds__(kThreads) grouped_q4_kernel(GroupedArgs a) {
  extern __shared__ float4 sm[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rs = lane / LPR, gl = lane % LPR;
  constexpr int RPP = 32 / LPR;                  // rows per warp pass
  constexpr int RPW = NR * RPP;                  // rows per warp
  constexpr int RPT = RPW * (kThreads / 32);     // rows per tile
  const int n_act = *a.n_active;
  const int total = n_act * a.tiles_per_expert;
  for (int tile = blockIdx.x; tile < total; tile += gridDim.x) {
    const int e = a.active[tile / a.tiles_per_expert];
    const int rb = tile % a.tiles_per_expert;
    const bool sh = e == a.E;
    const vx_q4 B0 = sh ? a.s0 : a.b0;
    const Q4Ptr p0 = q4_expert(B0, sh ? 0 : e);
    Q4Ptr p1 = p0;
    if (GATEUP) {
      const vx_q4 B1 = sh ? a.s1 : a.b1;
      p1 = q4_expert(B1, sh ? 0 : e);
    }
    const int K = B0.in, N = B0.out, G = K >> 5, KW = K >> 3;
    const int row0 = rb * RPT;
    if (row0 >= N) continue;  // uniform over the CTA
    const int lo = a.offsets[e], hi = a.offsets[e + 1];
    float4* xs = sm;                                             // [kTN][8][G]
    float* xsum = reinterpret_cast<float*>(sm + kTN * 8 * G);    // [kTN][G]
    for (int c0 = lo; c0 < hi; c0 += kTN) {
      const int nt = min(kTN, hi - c0);
      __syncthreads();
      // Stage x: element j of group g goes to xs[t][j/4][g].(j%4), scaled
      // by 16^-(j%4) (exact: a power of two).
      for (int it = threadIdx.x; it < nt * G * 4; it += kThreads) {
        const int t = it / (G * 4), rem = it - t * (G * 4), g = rem >> 2, c = rem & 3;
        const int pos = c0 + t;
        const int64_t row = a.src_rows ? a.src_rows[pos] : pos;
        const uint4 raw = *reinterpret_cast<const uint4*>(a.x + row * a.ldx + g * 32 + c * 8);
        const float v0 = __uint_as_float(raw.x << 16), v1 = __uint_as_float(raw.x & 0xFFFF0000u);
        const float v2 = __uint_as_float(raw.y << 16), v3 = __uint_as_float(raw.y & 0xFFFF0000u);
        const float v4 = __uint_as_float(raw.z << 16), v5 = __uint_as_float(raw.z & 0xFFFF0000u);
        const float v6 = __uint_as_float(raw.w << 16), v7 = __uint_as_float(raw.w & 0xFFFF0000u);
        xs[(t * 8 + 2 * c) * G + g] = make_float4(v0, v1 * 0.0625f, v2 * 0.00390625f, v3 * 0.000244140625f);
        xs[(t * 8 + 2 * c + 1) * G + g] =
            make_float4(v4, v5 * 0.0625f, v6 * 0.00390625f, v7 * 0.000244140625f);
      }
      for (int it = threadIdx.x; it < nt * G; it += kThreads) {
        const int t = it / G, g = it - t * G;
        const int pos = c0 + t;
        const int64_t row = a.src_rows ? a.src_rows[pos] : pos;
        const uint16_t* xr = a.x + row * a.ldx + g * 32;
        float s = 0.f;
#pragma unroll 8
        for (int j = 0; j < 32; ++j) s += bf16_to_f32(xr[j]);
        xsum[t * G + g] = s;
      }
      __syncthreads();

      float acc0[NR][kTN], acc1[NR][kTN];
#pragma unroll
      for (int i = 0; i < NR; ++i)
#pragma unroll
        for (int t = 0; t < kTN; ++t) acc0[i][t] = acc1[i][t] = 0.f;

      for (int g = gl; g < G; g += LPR) {
        uint4 w0[NR], w1[NR];
        float s0[NR], b0[NR], s1[NR], b1[NR];
#pragma unroll
        for (int i = 0; i < NR; ++i) {
          const int row = row0 + warp * RPW + i * RPP + rs;
          if (row < N) {
            const int64_t r = row;
            w0[i] = __ldg(reinterpret_cast<const uint4*>(p0.w + r * KW) + g);
            s0[i] = bf16_to_f32(__ldg(p0.s + r * G + g));
            b0[i] = bf16_to_f32(__ldg(p0.b + r * G + g));
            if (GATEUP) {
              w1[i] = __ldg(reinterpret_cast<const uint4*>(p1.w + r * KW) + g);
              s1[i] = bf16_to_f32(__ldg(p1.s + r * G + g));
              b1[i] = bf16_to_f32(__ldg(p1.b + r * G + g));
            }
          } else {
            w0[i] = w1[i] = make_uint4(0, 0, 0, 0);
            s0[i] = b0[i] = s1[i] = b1[i] = 0.f;
          }
        }
#pragma unroll
        for (int t = 0; t < kTN; ++t) {
          if (t < nt) {
            float4 xv[8];
#pragma unroll
            for (int j4 = 0; j4 < 8; ++j4) xv[j4] = xs[(t * 8 + j4) * G + g];
            const float xsm = xsum[t * G + g];
#pragma unroll
            for (int i = 0; i < NR; ++i) {
              acc0[i][t] += fmaf(s0[i], q4_dot_group(w0[i], xv), b0[i] * xsm);
              if (GATEUP) acc1[i][t] += fmaf(s1[i], q4_dot_group(w1[i], xv), b1[i] * xsm);
            }
          }
        }
      }
#pragma unroll
      for (int i = 0; i < NR; ++i) {
#pragma unroll
        for (int t = 0; t < kTN; ++t) {
          acc0[i][t] = warp_sum<LPR>(acc0[i][t]);
          if (GATEUP) acc1[i][t] = warp_sum<LPR>(acc1[i][t]);
        }
      }
      if (gl == 0) {
#pragma unroll
        for (int i = 0; i < NR; ++i) {
          const int row = row0 + warp * RPW + i * RPP + rs;
          if (row >= N) continue;
#pragma unroll
          for (int t = 0; t < kTN; ++t) {
            if (t >= nt) continue;
            const int pos = c0 + t;
            const int64_t dst = a.dst_rows ? a.dst_rows[pos] : pos;
            float v;
            if (GATEUP) v = silu_mul_bf16(bf16r(acc0[i][t]), bf16r(acc1[i][t]));
            else v = acc0[i][t];
            a.out[dst * a.ldo + row] = f32_to_bf16(v);
          }
        }
      }
    }
  }
}

template <int LPR, int NR, bool GATEUP>
static cudaError_t launch_t(const GroupedArgs& a0, int max_active, int max_out, int max_in,
                            cudaStream_t st) {
  constexpr int RPT = NR * (32 / LPR) * (kThreads / 32);
  GroupedArgs a = a0;
  a.tiles_per_expert = (max_out + RPT - 1) / RPT;
  const int G = max_in / 32;
  const size_t smem = size_t(kTN) * 8 * G * sizeof(float4) + size_t(kTN) * G * sizeof(float);
  auto kern = grouped_q4_kernel<LPR, NR, GATEUP>;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e != cudaSuccess) return e;
  }
  const int64_t tiles = int64_t(max_active) * a.tiles_per_expert;
  const int grid = int(tiles < int64_t(sm_count()) * 4 ? tiles : int64_t(sm_count()) * 4);
  if (grid <= 0) return cudaSuccess;
  kern<<<grid, kThreads, smem, st>>>(a);
  return cudaGetLastError();
}

template <bool GATEUP>
static cudaError_t launch_mode(const GroupedArgs& a, int max_active, int max_out, int max_in,
                               cudaStream_t st) {
  const int G = max_in / 32;
  if (G >= 32) return launch_t<32, 2, GATEUP>(a, max_active, max_out, max_in, st);
  if (G >= 16) return launch_t<16, 2, GATEUP>(a, max_active, max_out, max_in, st);
  if (G >= 8) return launch_t<8, 2, GATEUP>(a, max_active, max_out, max_in, st);
  if (G >= 4) return launch_t<4, 2, GATEUP>(a, max_active, max_out, max_in, st);
  return launch_t<1, 1, GATEUP>(a, max_active, max_out, max_in, st);
}

cudaError_t launch_grouped(GroupedMode mode, const GroupedArgs& a, int max_active, int max_out,
                           int max_in, cudaStream_t st) {
  if (mode == kGateUpSwiGLU) return launch_mode<true>(a, max_active, max_out, max_in, st);
  return launch_mode<false>(a, max_active, max_out, max_in, st);
}

}  // namespace vx
