// Router of the MoE block (models/flashnext/adaptive_topk.py:59-65,
// :257-265; compiled.py:60-70):
//   logits = bf16(x . Wg^T)                 unquantised bf16 gate
//   p = softmax(logits, precise)            float32 math, bf16 out
//   inds = top-k (logit desc, id asc)       see the tie rule below
//   scores = p[inds], mass = sum(scores)    bf16
//   weights = scores / mass                 renorm at blend 1.0
//   sg = sigmoid(shared_expert_gate(x))     Q4 row, bf16 sigmoid
//
// Tie rule: MLX's argpartition leaves the order of equal probabilities open.
// The kernel ranks by the bf16 logit, then the lower expert id.  Softmax is
// monotone, so this is always a valid top-k of the probabilities and it does
// not depend on how exp rounds.
#include "vx_common.cuh"
#include "vx_launch.h"

namespace vx {

// ---- logits: one warp per expert row, 8 tokens per pass ------------------
constexpr int kRouterTok = 8;

__global__ void __launch_bounds__(256) router_logits_kernel(const uint16_t* __restrict__ x, int T,
                                                            const uint16_t* __restrict__ wg, int E,
                                                            int K, uint16_t* __restrict__ logits) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int e = blockIdx.x * 8 + warp;
  if (e >= E) return;
  const uint16_t* wr = wg + int64_t(e) * K;
  for (int t0 = 0; t0 < T; t0 += kRouterTok) {
    const int nt = min(kRouterTok, T - t0);
    float acc[kRouterTok];
#pragma unroll
    for (int t = 0; t < kRouterTok; ++t) acc[t] = 0.f;
    for (int k0 = lane * 8; k0 < K; k0 += 256) {
      const uint4 wv = __ldg(reinterpret_cast<const uint4*>(wr + k0));
      float w[8] = {__uint_as_float(wv.x << 16), __uint_as_float(wv.x & 0xFFFF0000u),
                    __uint_as_float(wv.y << 16), __uint_as_float(wv.y & 0xFFFF0000u),
                    __uint_as_float(wv.z << 16), __uint_as_float(wv.z & 0xFFFF0000u),
                    __uint_as_float(wv.w << 16), __uint_as_float(wv.w & 0xFFFF0000u)};
#pragma unroll
      for (int t = 0; t < kRouterTok; ++t) {
        if (t < nt) {
          const uint4 xv = __ldg(reinterpret_cast<const uint4*>(x + int64_t(t0 + t) * K + k0));
          float a = acc[t];
          a = fmaf(__uint_as_float(xv.x << 16), w[0], a);
          a = fmaf(__uint_as_float(xv.x & 0xFFFF0000u), w[1], a);
          a = fmaf(__uint_as_float(xv.y << 16), w[2], a);
          a = fmaf(__uint_as_float(xv.y & 0xFFFF0000u), w[3], a);
          a = fmaf(__uint_as_float(xv.z << 16), w[4], a);
          a = fmaf(__uint_as_float(xv.z & 0xFFFF0000u), w[5], a);
          a = fmaf(__uint_as_float(xv.w << 16), w[6], a);
          a = fmaf(__uint_as_float(xv.w & 0xFFFF0000u), w[7], a);
          acc[t] = a;
        }
      }
    }
#pragma unroll
    for (int t = 0; t < kRouterTok; ++t) {
      const float v = warp_sum<32>(acc[t]);
      if (lane == 0 && t < nt) logits[int64_t(t0 + t) * E + e] = f32_to_bf16(v);
    }
  }
}

cudaError_t launch_router_logits(const uint16_t* x, int T, const uint16_t* wg, int E, int K,
                                 uint16_t* logits, cudaStream_t st) {
  if (T == 0) return cudaSuccess;
  router_logits_kernel<<<(E + 7) / 8, 256, 0, st>>>(x, T, wg, E, K, logits);
  return cudaGetLastError();
}

// ---- shared expert gate: one warp per token, Q4 row of width K ------------
__global__ void __launch_bounds__(256) shared_gate_kernel(const uint16_t* __restrict__ x, int T,
                                                          vx_q4 seg, uint16_t* __restrict__ sg) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x * 8 + warp;
  if (t >= T) return;
  const int K = seg.in, G = K / 32;
  const uint16_t* xr = x + int64_t(t) * K;
  float acc = 0.f;
  for (int g = lane; g < G; g += 32) {
    const uint4 w = __ldg(reinterpret_cast<const uint4*>(seg.w) + g);
    const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
    float q = 0.f, xs = 0.f;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        const float xv = bf16_to_f32(xr[g * 32 + c * 8 + n]);
        q = fmaf(float(nibble(ws[c], n)), xv, q);
        xs += xv;
      }
    }
    acc += fmaf(bf16_to_f32(seg.scales[g]), q, bf16_to_f32(seg.biases[g]) * xs);
  }
  acc = warp_sum<32>(acc);
  if (lane == 0) sg[t] = f32_to_bf16(sigmoid_bf16(bf16r(acc)));
}

cudaError_t launch_shared_gate(const uint16_t* x, int T, const vx_q4& seg, uint16_t* sg,
                               cudaStream_t st) {
  if (T == 0) return cudaSuccess;
  shared_gate_kernel<<<(T + 7) / 8, 256, 0, st>>>(x, T, seg, sg);
  return cudaGetLastError();
}

// ---- softmax + top-k + renorm: one warp per token --------------------------
constexpr int kMaxPer = 32;   // E <= 1024
constexpr int kMaxK = 16;

template <int PER>
__global__ void __launch_bounds__(256) softmax_topk_kernel(const uint16_t* __restrict__ logits,
                                                           int T, int E, int k,
                                                           int32_t* __restrict__ inds,
                                                           uint16_t* __restrict__ scores,
                                                           uint16_t* __restrict__ weights,
                                                           uint16_t* __restrict__ mass) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x * 8 + warp;
  if (t >= T) return;
  const uint16_t* lr = logits + int64_t(t) * E;
  float l[PER];
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    const int e = lane + 32 * j;
    l[j] = e < E ? bf16_to_f32(lr[e]) : -INFINITY;
  }
  float m = -INFINITY;
#pragma unroll
  for (int j = 0; j < PER; ++j) m = fmaxf(m, l[j]);
  m = warp_max(m);
  float ex[PER];
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    ex[j] = (lane + 32 * j < E) ? expf(__fsub_rn(l[j], m)) : 0.f;
    s += ex[j];
  }
  s = warp_sum<32>(s);
  const float inv = __fdiv_rn(1.0f, s);

  uint32_t taken = 0;
  int sel_i[kMaxK];
  float sel_p[kMaxK];
  for (int r = 0; r < k; ++r) {
    float bv = -INFINITY;
    int bi = 0x7FFFFFFF;
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      const int e = lane + 32 * j;
      if (e < E && !((taken >> j) & 1u) && (l[j] > bv || (l[j] == bv && e < bi))) {
        bv = l[j];
        bi = e;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xFFFFFFFFu, bv, o);
      const int oi = __shfl_xor_sync(0xFFFFFFFFu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
    const int owner = bi & 31, jj = bi >> 5;
    float mine = 0.f;
#pragma unroll
    for (int j = 0; j < PER; ++j)
      if (j == jj) mine = ex[j];
    const float ew = __shfl_sync(0xFFFFFFFFu, mine, owner);
    if (lane == owner) taken |= 1u << jj;
    if (r < kMaxK) {
      sel_i[r] = bi;
      sel_p[r] = bf16r(__fmul_rn(ew, inv));
    }
  }
  // mass and renorm (blend 1.0): norm = mass + 1.0*(sum - mass), in bf16.
  float tot = 0.f;
  for (int r = 0; r < k; ++r) tot = __fadd_rn(tot, sel_p[r]);
  const float msum = bf16r(tot);
  const float sel_sum = msum;
  const float diff = bf16r(__fsub_rn(sel_sum, msum));
  const float norm = bf16r(__fadd_rn(msum, bf16r(diff)));
  for (int r = lane; r < k; r += 32) {
    // r is warp-uniform per lane: pick the lane's slot from the arrays
    float p = 0.f;
    int id = 0;
    for (int q = 0; q < k; ++q)
      if (q == r) { p = sel_p[q]; id = sel_i[q]; }
    inds[int64_t(t) * k + r] = id;
    if (scores) scores[int64_t(t) * k + r] = f32_to_bf16(p);
    weights[int64_t(t) * k + r] = f32_to_bf16(bf16r(__fdiv_rn(p, norm)));
  }
  if (mass && lane == 0) mass[t] = f32_to_bf16(msum);
}

cudaError_t launch_softmax_topk(const uint16_t* logits, int T, int E, int k, int32_t* inds,
                                uint16_t* scores, uint16_t* weights, uint16_t* mass,
                                cudaStream_t st) {
  if (T == 0) return cudaSuccess;
  const int per = (E + 31) / 32;
  const int grid = (T + 7) / 8;
  if (per <= 4) softmax_topk_kernel<4><<<grid, 256, 0, st>>>(logits, T, E, k, inds, scores, weights, mass);
  else if (per <= 8) softmax_topk_kernel<8><<<grid, 256, 0, st>>>(logits, T, E, k, inds, scores, weights, mass);
  else if (per <= 16) softmax_topk_kernel<16><<<grid, 256, 0, st>>>(logits, T, E, k, inds, scores, weights, mass);
  else softmax_topk_kernel<32><<<grid, 256, 0, st>>>(logits, T, E, k, inds, scores, weights, mass);
  return cudaGetLastError();
}

}  // namespace vx
