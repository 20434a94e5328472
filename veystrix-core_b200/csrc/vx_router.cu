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
#include <type_traits>

#include "vx_async.cuh"
#include "vx_common.cuh"
#include "vx_launch.h"
#include "vx_perm_small.cuh"
#include "vx_topk.cuh"

namespace vx {

// ---- logits on the tensor pipe ---------------------------------------------
// A CTA owns 16 experts x 8 tokens; its kRouterSlices warps split K and meet
// in shared memory.  Lane (g, c) loads 16 bytes (8 bf16) of expert rows g and
// g+8 and of token g's x at the same k offset 8c: the same k permutation on
// both operands, so two m16n8k16 MMAs consume one 16-byte load per operand
// with no shuffling.  float32 accumulation, bf16 logits.
constexpr int kRouterSlices = 8;

__global__ void __launch_bounds__(32 * kRouterSlices) router_logits_kernel(
    const uint16_t* __restrict__ x, int T, const uint16_t* __restrict__ wg, int E, int K,
    uint16_t* __restrict__ logits) {
  __shared__ float red[kRouterSlices][32][4];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;
  const int e0 = blockIdx.x * 16, t0 = blockIdx.y * 8;
  const int ea = e0 + g, eb = e0 + g + 8, tx = t0 + g;
  const uint16_t* ra = wg + int64_t(ea < E ? ea : 0) * K;
  const uint16_t* rb = wg + int64_t(eb < E ? eb : 0) * K;
  const uint16_t* rx = x + int64_t(tx < T ? tx : 0) * K;
  const int steps = K / 32;
  const int per = (steps + kRouterSlices - 1) / kRouterSlices;
  const int s0 = warp * per, s1 = min(steps, s0 + per);
  float d[4] = {0.f, 0.f, 0.f, 0.f};
  for (int s = s0; s < s1; ++s) {
    const int k = s * 32 + c * 8;
    const uint4 wa = ea < E ? ldg_keep(ra + k) : make_uint4(0, 0, 0, 0);
    const uint4 wb = eb < E ? ldg_keep(rb + k) : make_uint4(0, 0, 0, 0);
    const uint4 xb = tx < T ? __ldg(reinterpret_cast<const uint4*>(rx + k)) : make_uint4(0, 0, 0, 0);
    mma16816(d, wa.x, wb.x, wa.y, wb.y, xb.x, xb.y);
    mma16816(d, wa.z, wb.z, wa.w, wb.w, xb.z, xb.w);
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) red[warp][lane][i] = d[i];
  __syncthreads();
  if (warp == 0) {
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    for (int w = 0; w < kRouterSlices; ++w)
#pragma unroll
      for (int i = 0; i < 4; ++i) v[i] += red[w][lane][i];
    // D[g][2c], D[g][2c+1], D[g+8][2c], D[g+8][2c+1]: (expert, token)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int e = (i < 2) ? ea : eb;
      const int t = t0 + 2 * c + (i & 1);
      if (e < E && t < T) logits[int64_t(t) * E + e] = f32_to_bf16(v[i]);
    }
  }
}

cudaError_t launch_router_logits(const uint16_t* x, int T, const uint16_t* wg, int E, int K,
                                 uint16_t* logits, cudaStream_t st) {
  if (T == 0) return cudaSuccess;
  dim3 grid((E + 15) / 16, (T + 7) / 8);
  router_logits_kernel<<<grid, 32 * kRouterSlices, 0, st>>>(x, T, wg, E, K, logits);
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
      const uint4 xv = __ldg(reinterpret_cast<const uint4*>(xr + g * 32 + c * 8));
      const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        const float v = __uint_as_float((n & 1) ? (xw[n >> 1] & 0xFFFF0000u) : (xw[n >> 1] << 16));
        q = fmaf(float(nibble(ws[c], n)), v, q);
        xs += v;
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

template <int PER>
__global__ void __launch_bounds__(256) softmax_topk_kernel(const uint16_t* __restrict__ logits,
                                                           int T, int E, int k,
                                                           int32_t* __restrict__ inds,
                                                           uint16_t* __restrict__ scores,
                                                           uint16_t* __restrict__ weights,
                                                           uint16_t* __restrict__ mass, double keep_mass,
                                                           int keep_min) {
  const int t = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (t >= T) return;
  topk_row<PER, false>(logits + int64_t(t) * E, E, k, inds + int64_t(t) * k,
                       scores ? scores + int64_t(t) * k : nullptr, weights + int64_t(t) * k,
                       mass ? mass + t : nullptr, keep_mass, keep_min);
}

template <class F>
static void per_width(int E, F&& f) {
  const int per = (E + 31) / 32;
  if (per <= 4) f(std::integral_constant<int, 4>());
  else if (per <= 8) f(std::integral_constant<int, 8>());
  else if (per <= 16) f(std::integral_constant<int, 16>());
  else f(std::integral_constant<int, 32>());
}

cudaError_t launch_softmax_topk(const uint16_t* logits, int T, int E, int k, int32_t* inds,
                                uint16_t* scores, uint16_t* weights, uint16_t* mass,
                                cudaStream_t st, double keep_mass, int keep_min) {
  if (T == 0) return cudaSuccess;
  if (k > kMaxK) return cudaErrorInvalidValue;
  const int grid = (T + 7) / 8;
  per_width(E, [&](auto per) {
    softmax_topk_kernel<decltype(per)::value>
        <<<grid, 256, 0, st>>>(logits, T, E, k, inds, scores, weights, mass, keep_mass, keep_min);
  });
  return cudaGetLastError();
}

// ---- the fused router: logits, then top-k by the last CTA of each token
// block, and the shared-expert gate in an extra CTA column ----------------
// CTA (eb, tb), eb < nEB: the 16 x 8 logits tile of router_logits_kernel,
// then an acquire-release arrival on the token block's counter; the CTA that
// arrives last (every tile is then visible to it) runs softmax/top-k for
// the block's 8 tokens (one warp each) and resets the counter.  CTA eb == nEB
// computes sigmoid(shared_expert_gate(x)) for the 8 tokens.  With perm.order
// set, the token blocks' last CTAs take a second ticket (counter nTB) and the
// last of them sorts all T*k routes by expert (perm_small).  The counters
// (one per token block, plus the second ticket) must be zero at launch.
template <int PER>
__global__ void __launch_bounds__(32 * kRouterSlices) router_fused_kernel(
    const uint16_t* __restrict__ x, int T, const uint16_t* __restrict__ wg, int E, int K, int k, vx_q4 seg,
    uint16_t* __restrict__ logits, int32_t* __restrict__ inds, uint16_t* __restrict__ weights,
    uint16_t* __restrict__ sg, int32_t* __restrict__ counters, PermSmallArgs perm,
    const uint16_t* __restrict__ bias, double keep_mass, int keep_min) {
  chain_begin();
  const int nEB = (E + 15) / 16;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t0 = blockIdx.y * 8;
  if (int(blockIdx.x) == nEB) {
    // shared expert gate: warp w -> token t0 + w
    const int t = t0 + warp;
    if (!sg || !seg.w || t >= T) return;
    const int G = K / 32;
    const uint16_t* xr = x + int64_t(t) * K;
    float acc = 0.f;
    for (int g = lane; g < G; g += 32) {
      const uint4 w = __ldg(reinterpret_cast<const uint4*>(seg.w) + g);
      const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
      float q = 0.f, xs = 0.f;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const uint4 xv = __ldg(reinterpret_cast<const uint4*>(xr + g * 32 + c * 8));
        const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
        for (int n = 0; n < 8; ++n) {
          const float v = __uint_as_float((n & 1) ? (xw[n >> 1] & 0xFFFF0000u) : (xw[n >> 1] << 16));
          q = fmaf(float(nibble(ws[c], n)), v, q);
          xs += v;
        }
      }
      acc += fmaf(bf16_to_f32(seg.scales[g]), q, bf16_to_f32(seg.biases[g]) * xs);
    }
    acc = warp_sum<32>(acc);
    if (lane == 0) sg[t] = f32_to_bf16(sigmoid_bf16(bf16r(acc)));
    return;
  }
  __shared__ float red[kRouterSlices][32][4];
  __shared__ int s_last;
  const int g = lane >> 2, c = lane & 3;
  const int e0 = blockIdx.x * 16;
  const int ea = e0 + g, eb = e0 + g + 8, tx = t0 + g;
  const uint16_t* ra = wg + int64_t(ea < E ? ea : 0) * K;
  const uint16_t* rb = wg + int64_t(eb < E ? eb : 0) * K;
  const uint16_t* rx = x + int64_t(tx < T ? tx : 0) * K;
  const int steps = K / 32;
  const int per = (steps + kRouterSlices - 1) / kRouterSlices;
  const int s0 = warp * per, s1 = min(steps, s0 + per);
  float d[4] = {0.f, 0.f, 0.f, 0.f};
  // All loads of a batch of steps are issued before its MMAs (same MMA
  // order as one step at a time), so a warp keeps up to 6 KiB in flight and
  // a CTA fetches its 64 KiB of router rows in about one memory round trip.
  constexpr int kBatch = 8;
  const uint4 zero = make_uint4(0, 0, 0, 0);
  for (int sb = s0; sb < s1; sb += kBatch) {
    uint4 wa[kBatch], wb[kBatch], xb[kBatch];
#pragma unroll
    for (int i = 0; i < kBatch; ++i) {
      const int s = sb + i;
      const int kk = s * 32 + c * 8;
      wa[i] = (s < s1 && ea < E) ? ldg_keep(ra + kk) : zero;
      wb[i] = (s < s1 && eb < E) ? ldg_keep(rb + kk) : zero;
      xb[i] = (s < s1 && tx < T) ? __ldg(reinterpret_cast<const uint4*>(rx + kk)) : zero;
    }
#pragma unroll
    for (int i = 0; i < kBatch; ++i) {
      if (sb + i < s1) {
        mma16816(d, wa[i].x, wb[i].x, wa[i].y, wb[i].y, xb[i].x, xb[i].y);
        mma16816(d, wa[i].z, wb[i].z, wa[i].w, wb[i].w, xb[i].z, xb[i].w);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) red[warp][lane][i] = d[i];
  __syncthreads();
  if (warp == 0) {
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    for (int w = 0; w < kRouterSlices; ++w)
#pragma unroll
      for (int i = 0; i < 4; ++i) v[i] += red[w][lane][i];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int e = (i < 2) ? ea : eb;
      const int t = t0 + 2 * c + (i & 1);
      if (e < E && t < T) {
        float l = bf16r(v[i]);
        if (bias) l = bf16r(__fadd_rn(l, bf16_to_f32(bias[e])));   // bf16 logits + bf16 bias
        logits[int64_t(t) * E + e] = f32_to_bf16(l);
      }
    }
  }
  // Arrival: the barrier orders the tile's stores before thread 0's
  // acquire-release add (release of this tile; for the last CTA, acquire of
  // every other tile, passed to its threads by the second barrier).  No
  // separate fence: a full fence here cost microseconds on the critical path.
  __syncthreads();
  if (threadIdx.x == 0) {
    int prev;
    asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;"
                 : "=r"(prev)
                 : "l"(counters + blockIdx.y)
                 : "memory");
    s_last = prev == nEB - 1;
  }
  __syncthreads();
  if (!s_last) return;
  const int t = t0 + warp;
  if (t < T)
    topk_row<PER, true>(logits + int64_t(t) * E, E, k, inds + int64_t(t) * k, nullptr, weights + int64_t(t) * k,
                        nullptr, keep_mass, keep_min);
  if (perm.order) {
    // decode-sized batch: the last token block to finish also sorts the
    // routes by expert, saving the permutation's own launch.  Second arrival
    // (over token blocks, counter gridDim.y), ordered like the first: the
    // barrier puts this block's ids before thread 0's acquire-release add.
    __shared__ int s_final;
    __syncthreads();   // every token's ids of this block are written
    if (threadIdx.x == 0) {
      int prev = 0;
      if (gridDim.y > 1)
        asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;"
                     : "=r"(prev)
                     : "l"(counters + gridDim.y)
                     : "memory");
      s_final = prev == int(gridDim.y) - 1;
    }
    __syncthreads();
    if (s_final) {
      perm_small(perm, inds, T * k);
      if (threadIdx.x == 0) counters[gridDim.y] = 0;
    }
  }
  if (threadIdx.x == 0) counters[blockIdx.y] = 0;
}

// ---- prefill-sized batches: logits of a 64-expert x 64-token tile per CTA --
// The fused kernel's tiles (16 experts x 8 tokens) re-read the router matrix
// from L2 once per 8 tokens: at 2,048 tokens that is 512 MB of L2 traffic for
// a 2 MB matrix.  Here a CTA stages 64 expert rows and 64 token rows, four
// 32-input steps at a time (cp.async, double-buffered, 68 KB: three CTAs per
// SM), and reuses each row 4 or 16 times from shared memory.  The arithmetic
// is the fused kernel's, in its order: K cut into the same 8 slices of `per`
// steps, each slice's MMAs (the same fragments: lane (g, c) takes inputs
// 8c..8c+7 of a step from expert rows g, g+8 and token row g) summed from
// zero, the slice sums (empty slices' zeros included) added in slice order,
// then the bf16 rounding and the bias - so the logits equal the fused
// kernel's bit for bit.
constexpr int kRtRows = 64;   // experts and tokens per CTA tile
constexpr int kRtSteps = 4;   // 32-input steps per staged chunk
constexpr int kRtLd = kRtSteps * 32 + 8;   // bf16 per staged row (16-byte pad)
constexpr size_t kRtSmem = size_t(2) * 2 * kRtRows * kRtLd * sizeof(uint16_t);

__global__ void __launch_bounds__(256) router_tiled_kernel(const uint16_t* __restrict__ x, int T,
                                                           const uint16_t* __restrict__ wg, int E, int K,
                                                           uint16_t* __restrict__ logits,
                                                           const uint16_t* __restrict__ bias) {
  chain_begin();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t0 = blockIdx.y * kRtRows, e0 = blockIdx.x * kRtRows;
  extern __shared__ __align__(16) unsigned char rt_smem[];
  uint16_t* sw = reinterpret_cast<uint16_t*>(rt_smem);   // [2][64][kRtLd] expert rows
  uint16_t* sx = sw + 2 * kRtRows * kRtLd;               // [2][64][kRtLd] token rows
  const int steps = K / 32;
  const int per = (steps + kRouterSlices - 1) / kRouterSlices;   // steps per slice
  // stage steps c0 .. c0+n-1 into buffer b
  auto load = [&](int c0, int n, int b) {
    const int chunks = n * 4;   // 16-byte pieces per row
    for (int idx = threadIdx.x; idx < kRtRows * chunks; idx += blockDim.x) {
      const int r = idx / chunks, ch = idx - r * chunks;
      const int e = e0 + r, t = t0 + r;
      const int k = c0 * 32 + ch * 8;
      cp16_if(smem_u32(sw + (b * kRtRows + r) * kRtLd + ch * 8), e < E ? wg + int64_t(e) * K + k : wg,
              e < E ? 16 : 0, true);
      cp16_if(smem_u32(sx + (b * kRtRows + r) * kRtLd + ch * 8), t < T ? x + int64_t(t) * K + k : x,
              t < T ? 16 : 0, true);
    }
  };
  // the chunk after (sl, c0): the next steps of the slice, else the first
  // step of the next slice that has any (sl = kRouterSlices: none)
  auto next_chunk = [&](int& sl, int& c0) {
    c0 += kRtSteps;
    if (c0 < min(steps, (sl + 1) * per)) return;
    for (++sl; sl < kRouterSlices && sl * per >= steps; ++sl) {
    }
    c0 = sl * per;
  };
  const int g = lane >> 2, c = lane & 3;
  const int ew = (warp & 3) * 16, tw = (warp >> 2) * 32;
  float tot[4][4], part[4][4];
#pragma unroll
  for (int j = 0; j < 4; ++j)
#pragma unroll
    for (int i = 0; i < 4; ++i) tot[j][i] = part[j][i] = 0.f;
  if (steps > 0) load(0, min(kRtSteps, per), 0);
  cp_commit();
  int q = 0;
  for (int sl = 0; sl < kRouterSlices; ++sl) {
    const int s_end = min(steps, (sl + 1) * per);
    for (int c0 = sl * per; c0 < s_end; c0 += kRtSteps, ++q) {
      int nsl = sl, nc0 = c0;
      next_chunk(nsl, nc0);
      if (nsl < kRouterSlices) load(nc0, min(kRtSteps, min(steps, (nsl + 1) * per) - nc0), (q + 1) & 1);
      cp_commit();
      cp_wait<1>();
      __syncthreads();
      const int b = q & 1;
      const int ns = min(kRtSteps, s_end - c0);
      const uint16_t* wa_row = sw + (b * kRtRows + ew + g) * kRtLd + c * 8;
      const uint16_t* wb_row = wa_row + 8 * kRtLd;
      const uint16_t* x_row = sx + (b * kRtRows + tw + g) * kRtLd + c * 8;
      for (int ls = 0; ls < ns; ++ls) {
        const uint4 wa = lds128(smem_u32(wa_row + ls * 32));
        const uint4 wb = lds128(smem_u32(wb_row + ls * 32));
        uint4 xb[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) xb[j] = lds128(smem_u32(x_row + j * 8 * kRtLd + ls * 32));
#pragma unroll
        for (int j = 0; j < 4; ++j) mma16816(part[j], wa.x, wb.x, wa.y, wb.y, xb[j].x, xb[j].y);
#pragma unroll
        for (int j = 0; j < 4; ++j) mma16816(part[j], wa.z, wb.z, wa.w, wb.w, xb[j].z, xb[j].w);
      }
      __syncthreads();   // the buffer is read out before a later load refills it
    }
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        tot[j][i] += part[j][i];
        part[j][i] = 0.f;
      }
  }
  // D[g][2c], D[g][2c+1], D[g+8][2c], D[g+8][2c+1] of each (16 experts, 8 tokens) tile
#pragma unroll
  for (int j = 0; j < 4; ++j)
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int e = e0 + ew + g + (i < 2 ? 0 : 8);
      const int t = t0 + tw + 8 * j + 2 * c + (i & 1);
      if (e < E && t < T) {
        float l = bf16r(tot[j][i]);
        if (bias) l = bf16r(__fadd_rn(l, bf16_to_f32(bias[e])));   // bf16 logits + bf16 bias
        logits[int64_t(t) * E + e] = f32_to_bf16(l);
      }
    }
}

bool router_tiled_fits(int T, int K) { return T >= kRouterTiledMinT && K <= 2048 && K % 32 == 0; }

cudaError_t launch_router_tiled(const uint16_t* x, int T, const uint16_t* wg, int E, int K, int k,
                                const vx_q4* seg, uint16_t* logits, int32_t* inds, uint16_t* weights,
                                uint16_t* sg, const uint16_t* bias, cudaStream_t st, double keep_mass,
                                int keep_min) {
  if (T == 0) return cudaSuccess;
  if (k > kMaxK || !router_tiled_fits(T, K)) return cudaErrorInvalidValue;
  cudaError_t e = cudaFuncSetAttribute(router_tiled_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       int(kRtSmem));
  if (e != cudaSuccess) return e;
  const dim3 grid((E + kRtRows - 1) / kRtRows, (T + kRtRows - 1) / kRtRows);
  e = launch_chained(router_tiled_kernel, grid, dim3(256), kRtSmem, st, x, T, wg, E, K, logits, bias);
  if (e == cudaSuccess)
    e = launch_softmax_topk(logits, T, E, k, inds, nullptr, weights, nullptr, st, keep_mass, keep_min);
  if (e == cudaSuccess && seg && sg) e = launch_shared_gate(x, T, *seg, sg, st);
  return e;
}

cudaError_t launch_router_fused(const uint16_t* x, int T, const uint16_t* wg, int E, int K, int k,
                                const vx_q4* seg, uint16_t* logits, int32_t* inds, uint16_t* weights,
                                uint16_t* sg, int32_t* counters, const PermSmallArgs* perm,
                                const uint16_t* bias, cudaStream_t st, bool counters_zeroed,
                                double keep_mass, int keep_min) {
  if (T == 0) return cudaSuccess;
  if (k > kMaxK) return cudaErrorInvalidValue;
  const int nTB = (T + 7) / 8, nEB = (E + 15) / 16;
  PermSmallArgs pa{};
  if (perm) {
    if (int64_t(T) * k > kPermSmall || E > kPermSmallMaxE) return cudaErrorInvalidValue;
    pa = *perm;
  }
  cudaError_t e = cudaSuccess;
  if (!counters_zeroed) {
    e = cudaMemsetAsync(counters, 0, size_t(router_counters(T)) * sizeof(int32_t), st);
    if (e != cudaSuccess) return e;
  }
  vx_q4 q{};
  if (seg) q = *seg;
  dim3 grid(nEB + 1, nTB);
  per_width(E, [&](auto per) {
    e = launch_chained(router_fused_kernel<decltype(per)::value>, grid, dim3(32 * kRouterSlices), 0, st, x, T,
                       wg, E, K, k, q, logits, inds, weights, sg, counters, pa, bias, keep_mass, keep_min);
  });
  return e;
}

}  // namespace vx
