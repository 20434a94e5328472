// Combine, unpermute, RMSNorm and the small Q4/bf16 contract kernels.
#include "vx_common.cuh"
#include "vx_launch.h"

namespace vx {

// V consecutive bf16 values as float32 (V = 8: one 16-byte load; 2: 4 bytes).
template <int V>
VX_DEVICE void load_bf16(const uint16_t* p, float (&f)[V]) {
  if constexpr (V == 8) {
    const uint4 v = *reinterpret_cast<const uint4*>(p);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      f[2 * i] = __uint_as_float(w[i] << 16);
      f[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
    }
  } else {
    static_assert(V == 2, "2 or 8 values");
    const uint32_t v = *reinterpret_cast<const uint32_t*>(p);
    f[0] = __uint_as_float(v << 16);
    f[1] = __uint_as_float(v & 0xFFFF0000u);
  }
}

template <int V>
VX_DEVICE void store_bf16(uint16_t* p, const float (&f)[V]) {
  uint32_t w[V / 2];
#pragma unroll
  for (int i = 0; i < V / 2; ++i) w[i] = uint32_t(f32_to_bf16(f[2 * i])) | (uint32_t(f32_to_bf16(f[2 * i + 1])) << 16);
  if constexpr (V == 8)
    *reinterpret_cast<uint4*>(p) = make_uint4(w[0], w[1], w[2], w[3]);
  else
    *reinterpret_cast<uint32_t*>(p) = w[0];
}

// a[i] = sum over the token's slots, in slot order, of bf16(yd[pos][c + i]) *
// score, each product and sum rounded (no fused multiply-add); slots with
// pos < 0 (dropped) add nothing.  The rows of up to kCombineBatch slots are
// loaded before any of them is added, so a thread keeps that many loads in
// flight instead of one.
constexpr int kCombineBatch = 8;

template <int V>
VX_DEVICE void slot_sum(const uint16_t* __restrict__ yd, int64_t ldy, const int32_t* __restrict__ inv,
                        const uint16_t* __restrict__ wts, int k, int c, float (&a)[V]) {
#pragma unroll
  for (int i = 0; i < V; ++i) a[i] = 0.f;
  for (int s0 = 0; s0 < k; s0 += kCombineBatch) {
    int pos[kCombineBatch];
    float w[kCombineBatch], v[kCombineBatch][V];
#pragma unroll
    for (int j = 0; j < kCombineBatch; ++j) {
      pos[j] = s0 + j < k ? inv[s0 + j] : -1;
      w[j] = pos[j] >= 0 ? bf16_to_f32(wts[s0 + j]) : 0.f;
    }
#pragma unroll
    for (int j = 0; j < kCombineBatch; ++j) {
      if (pos[j] >= 0) {
        load_bf16<V>(yd + int64_t(pos[j]) * ldy + c, v[j]);
      } else {
#pragma unroll
        for (int i = 0; i < V; ++i) v[j][i] = 0.f;
      }
    }
#pragma unroll
    for (int j = 0; j < kCombineBatch; ++j)
      if (pos[j] >= 0)
#pragma unroll
        for (int i = 0; i < V; ++i) a[i] = __fadd_rn(a[i], __fmul_rn(v[j][i], w[j]));
  }
}

// Score-weighted combine of the routed outputs, in the order of the fused
// down+combine kernel of the reference (metal_runtime.py:315-334, patched
// helpers :404-410): every slot's output is already bf16; it is multiplied
// by its score and accumulated in float32 in slot order without fused
// multiply-add; the sum is rounded to bf16, then the shared component is
// added in float32 and the result rounded to bf16.
// One thread per V consecutive outputs of token t (blockIdx.x).
template <int V>
__global__ void __launch_bounds__(256) combine_kernel(
    const uint16_t* __restrict__ yd, int64_t ldy, const int32_t* __restrict__ inverse,
    const uint16_t* __restrict__ weights, int T, int k, int d, int mode,
    const int32_t* __restrict__ offsets, int E, const uint16_t* __restrict__ sg,
    const uint16_t* __restrict__ shared_y, const uint16_t* __restrict__ shared,
    const uint16_t* __restrict__ shared_gate, uint16_t* __restrict__ y) {
  chain_begin();
  const int t = blockIdx.x;
  const int c = (blockIdx.y * blockDim.x + threadIdx.x) * V;   // rows on x: no 65,535 limit
  if (c >= d) return;
  float a[V], r[V];
  slot_sum<V>(yd, ldy, inverse + int64_t(t) * k, weights + int64_t(t) * k, k, c, a);
#pragma unroll
  for (int i = 0; i < V; ++i) r[i] = bf16r(a[i]);
  if (mode != kSharedNone) {
    float sv[V];
    if (mode == kSharedY) {
      load_bf16<V>(shared_y + int64_t(t) * d + c, sv);
    } else {
      const uint16_t* srow;
      float gate;
      if (mode == kSharedInternal) {
        srow = yd + int64_t(offsets[E] + t) * ldy;
        gate = bf16_to_f32(sg[t]);
      } else {
        srow = shared + int64_t(t) * d;
        gate = bf16_to_f32(shared_gate[t]);
      }
      load_bf16<V>(srow + c, sv);
#pragma unroll
      for (int i = 0; i < V; ++i) sv[i] = bf16r(__fmul_rn(sv[i], gate));
    }
#pragma unroll
    for (int i = 0; i < V; ++i) r[i] = bf16r(__fadd_rn(r[i], sv[i]));
  }
  store_bf16<V>(y + int64_t(t) * d + c, r);
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

cudaError_t launch_combine(const uint16_t* yd, int64_t ldy, const int32_t* inverse,
                           const uint16_t* weights, int T, int k, int d, SharedMode mode,
                           const int32_t* offsets, int E, const uint16_t* sg,
                           const uint16_t* shared_y, const uint16_t* shared,
                           const uint16_t* shared_gate, uint16_t* y, cudaStream_t st) {
  if (T == 0) return cudaSuccess;
  // eight outputs per thread when every row the kernel reads or writes
  // starts on a 16-byte boundary and the batch still gives every SM two
  // CTAs (decode-sized batches keep two outputs per thread and more CTAs)
  const bool wide = d % 8 == 0 && ldy % 8 == 0 && aligned16(yd) && aligned16(y) &&
                    (!shared_y || aligned16(shared_y)) && (!shared || aligned16(shared)) &&
                    int64_t(T) * ((d / 8 + 255) / 256) >= 2 * int64_t(sm_count());
  if (wide)
    return launch_chained(combine_kernel<8>, dim3(T, (d / 8 + 255) / 256), dim3(256), 0, st, yd, ldy, inverse,
                          weights, T, k, d, int(mode), offsets, E, sg, shared_y, shared, shared_gate, y);
  return launch_chained(combine_kernel<2>, dim3(T, (d / 2 + 255) / 256), dim3(256), 0, st, yd, ldy, inverse,
                        weights, T, k, d, int(mode), offsets, E, sg, shared_y, shared, shared_gate, y);
}

// Activations for the grouped GEMV: B order and per-group sums.  One thread
// per 8-input block; the four threads of a quant group are adjacent lanes
// (K/8 is a multiple of 4), so the group sum is a two-step xor shuffle:
// (s0 + s1) + (s2 + s3), each s a left-to-right float32 sum of 8 inputs.
__global__ void xprep_kernel(const uint16_t* __restrict__ x, int64_t rows, int K,
                             uint16_t* __restrict__ xb, float* __restrict__ xs, int64_t ldxs) {
  chain_begin();
  const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  const int nb = K / 8;
  const int64_t n = rows * nb;
  const bool live = i < n;
  const int64_t r = live ? i / nb : 0;
  const int blk = live ? int(i - r * nb) : 0;
  uint4 v = make_uint4(0, 0, 0, 0);
  if (live) v = *reinterpret_cast<const uint4*>(x + r * K + blk * 8);
  float s = 0.f;
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    s += __uint_as_float(w[j] << 16);
    s += __uint_as_float(w[j] & 0xFFFF0000u);
  }
  s += __shfl_xor_sync(0xFFFFFFFFu, s, 1);
  s += __shfl_xor_sync(0xFFFFFFFFu, s, 2);
  if (!live) return;
  uint4 o;
  o.x = prmt(v.x, v.z, 0x5410);   // (x0, x4)
  o.y = prmt(v.x, v.z, 0x7632);   // (x1, x5)
  o.z = prmt(v.y, v.w, 0x5410);   // (x2, x6)
  o.w = prmt(v.y, v.w, 0x7632);   // (x3, x7)
  *reinterpret_cast<uint4*>(xb + r * K + blk * 8) = o;
  if ((blk & 3) == 0) {
    const int grp = blk >> 2;
    xs[r * ldxs + grp] = s;
    if (grp + 1 == K / 32 && (K / 32) < ldxs) xs[r * ldxs + grp + 1] = 0.f;
  }
}

cudaError_t launch_xprep(const uint16_t* x, int64_t rows, int K, uint16_t* xb, float* xs,
                         int64_t ldxs, cudaStream_t st) {
  const int64_t n = rows * (K / 8);
  if (n == 0) return cudaSuccess;
  return launch_chained(xprep_kernel, dim3(int((n + 255) / 256)), dim3(256), 0, st, x, rows, K, xb, xs,
                        ldxs);
}

// Float32 partial combine for expert parallelism: the same slot-order
// float32 sum as combine_kernel, left unrounded and without the shared part
// (the home rank adds the partials of all ranks, then rounds).
template <int V>
__global__ void __launch_bounds__(256) combine_partial_kernel(
    const uint16_t* __restrict__ yd, int64_t ldy, const int32_t* __restrict__ inverse,
    const uint16_t* __restrict__ weights, int k, int d, float* __restrict__ out) {
  chain_begin();
  const int t = blockIdx.x;
  const int c = (blockIdx.y * blockDim.x + threadIdx.x) * V;   // rows on x: no 65,535 limit
  if (c >= d) return;
  float a[V];
  slot_sum<V>(yd, ldy, inverse + int64_t(t) * k, weights + int64_t(t) * k, k, c, a);
  float* o = out + int64_t(t) * d + c;
#pragma unroll
  for (int i = 0; i < V; i += 2) *reinterpret_cast<float2*>(o + i) = make_float2(a[i], a[i + 1]);
}

cudaError_t launch_combine_partial(const uint16_t* yd, int64_t ldy, const int32_t* inverse,
                                   const uint16_t* weights, int T, int k, int d, float* out,
                                   cudaStream_t st) {
  if (T == 0) return cudaSuccess;
  if (d % 8 == 0 && ldy % 8 == 0 && aligned16(yd) && aligned16(out) &&
      int64_t(T) * ((d / 8 + 255) / 256) >= 2 * int64_t(sm_count()))
    return launch_chained(combine_partial_kernel<8>, dim3(T, (d / 8 + 255) / 256), dim3(256), 0, st, yd, ldy,
                          inverse, weights, k, d, out);
  return launch_chained(combine_partial_kernel<2>, dim3(T, (d / 2 + 255) / 256), dim3(256), 0, st, yd, ldy,
                        inverse, weights, k, d, out);
}

// out[t, s, :] = yd[inverse[t*k+s], :]  (_scatter_unsort)
__global__ void unpermute_kernel(const uint16_t* __restrict__ yd, int64_t ldy,
                                 const int32_t* __restrict__ inverse, int k, int d,
                                 uint16_t* __restrict__ out) {
  chain_begin();
  const int64_t pair = blockIdx.x;
  const int c = (blockIdx.y * blockDim.x + threadIdx.x) * 2;   // rows on x: no 65,535 limit
  if (c >= d) return;
  const int pos = inverse[pair];
  uint32_t v = 0;
  if (pos >= 0) v = *reinterpret_cast<const uint32_t*>(yd + int64_t(pos) * ldy + c);
  *reinterpret_cast<uint32_t*>(out + pair * d + c) = v;
}

cudaError_t launch_unpermute(const uint16_t* yd, int64_t ldy, const int32_t* inverse, int T,
                             int k, int d, uint16_t* out, cudaStream_t st) {
  if (T == 0) return cudaSuccess;
  dim3 grid(T * k, (d / 2 + 255) / 256);
  return launch_chained(unpermute_kernel, grid, dim3(256), 0, st, yd, ldy, inverse, k, d, out);
}

// RMSNorm (patch_rmsnorm.py:96-120): y = bf16(x * (1/sqrt(mean(x^2)+eps)) * gain)
// with float32 arithmetic; one CTA per row.
__global__ void __launch_bounds__(256) rmsnorm_kernel(const uint16_t* __restrict__ x,
                                                      const uint16_t* __restrict__ gain, int d,
                                                      float eps, uint16_t* __restrict__ y) {
  chain_begin();
  const int64_t t = blockIdx.x;
  const uint16_t* xr = x + t * d;
  float s = 0.f;
  for (int i = threadIdx.x; i < d; i += blockDim.x) {
    const float v = bf16_to_f32(xr[i]);
    s = fmaf(v, v, s);
  }
  __shared__ float red[8];
  s = warp_sum<32>(s);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  float tot = 0.f;
  for (int w = 0; w < int(blockDim.x >> 5); ++w) tot += red[w];
  const float ms = __fdiv_rn(tot, float(d));
  const float r = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ms, eps)));
  for (int i = threadIdx.x; i < d; i += blockDim.x) {
    const float v = __fmul_rn(__fmul_rn(bf16_to_f32(xr[i]), r), bf16_to_f32(gain[i]));
    y[t * d + i] = f32_to_bf16(v);
  }
}

cudaError_t launch_rmsnorm(const uint16_t* x, const uint16_t* gain, int T, int d, float eps,
                           uint16_t* y, cudaStream_t st) {
  if (T == 0) return cudaSuccess;
  return launch_chained(rmsnorm_kernel, dim3(T), dim3(256), 0, st, x, gain, d, eps, y);
}

__global__ void swiglu_kernel(const uint16_t* __restrict__ g, const uint16_t* __restrict__ u,
                              uint16_t* __restrict__ out, int64_t n) {
  const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  out[i] = f32_to_bf16(silu_mul_bf16(bf16_to_f32(g[i]), bf16_to_f32(u[i])));
}

cudaError_t launch_swiglu(const uint16_t* g, const uint16_t* u, uint16_t* out, int64_t n,
                          cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  swiglu_kernel<<<int((n + 255) / 256), 256, 0, st>>>(g, u, out, n);
  return cudaGetLastError();
}

// Dequantise expert e: out[r, i] = scale*q + bias (scale*q is exact in fp32,
// so one rounding, metal_runtime.py:1026-1027).
__global__ void dequant_kernel(vx_q4 bank, int e, float* __restrict__ out) {
  const int64_t n = int64_t(bank.out) * bank.in;
  const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const Q4Ptr p = q4_expert(bank, e);
  const int64_t r = i / bank.in, k = i - r * bank.in;
  const uint32_t w = p.w[r * (bank.in / 8) + k / 8];
  const int64_t gi = r * (bank.in / bank.group_size) + k / bank.group_size;
  const float q = float(nibble(w, int(k & 7)));
  out[i] = __fadd_rn(__fmul_rn(bf16_to_f32(p.s[gi]), q), bf16_to_f32(p.b[gi]));
}

cudaError_t launch_dequant(const vx_q4& bank, int expert, float* out, cudaStream_t st) {
  const int64_t n = int64_t(bank.out) * bank.in;
  if (n == 0) return cudaSuccess;
  dequant_kernel<<<int((n + 255) / 256), 256, 0, st>>>(bank, expert, out);
  return cudaGetLastError();
}

// Combine of already projected values, the reference's generic helper
// (models/flashnext/metal_runtime.py:145-191): y[t] = sum_s out[t, sel(s)] *
// score[t, s], sel(s) = routes[t, s] when the outputs hold every expert (n_out
// rows per token), else the slot itself.  Products in the element type (bf16
// products rounded to bf16), summed in float32 in slot order, one rounding to
// the element type - what the array expression computes on bf16 or float32
// arrays.  Routes outside [0, n_out) contribute nothing and are counted in
// *err (may be null).
template <bool BF16>
__global__ void __launch_bounds__(256) weighted_combine_kernel(const void* __restrict__ outputs, int n_out,
                                                               const int32_t* __restrict__ routes,
                                                               const void* __restrict__ scores, int64_t T, int k,
                                                               int d, void* __restrict__ y, int32_t* err) {
  const int64_t t = blockIdx.x;
  const int col = blockIdx.y * blockDim.x + threadIdx.x;
  if (t >= T || col >= d) return;
  float acc = 0.f;
  for (int s = 0; s < k; ++s) {
    const int e = routes ? routes[t * k + s] : s;
    if (e < 0 || e >= n_out) {
      if (col == 0 && err) atomicAdd(err, 1);
      continue;
    }
    const int64_t i = (t * n_out + e) * int64_t(d) + col;
    if (BF16) {
      const float v = bf16_to_f32(static_cast<const uint16_t*>(outputs)[i]);
      const float w = bf16_to_f32(static_cast<const uint16_t*>(scores)[t * k + s]);
      acc = __fadd_rn(acc, bf16r(__fmul_rn(v, w)));
    } else {
      const float v = static_cast<const float*>(outputs)[i];
      const float w = static_cast<const float*>(scores)[t * k + s];
      acc = __fadd_rn(acc, __fmul_rn(v, w));
    }
  }
  if (BF16)
    static_cast<uint16_t*>(y)[t * d + col] = f32_to_bf16(acc);
  else
    static_cast<float*>(y)[t * d + col] = acc;
}

cudaError_t launch_weighted_combine(const void* outputs, int n_out, const int32_t* routes, const void* scores,
                                    int64_t T, int k, int d, bool bf16, void* y, int32_t* err,
                                    cudaStream_t st) {
  if (T == 0 || d == 0) return cudaSuccess;
  dim3 grid(unsigned(T), unsigned((d + 255) / 256));
  if (bf16)
    weighted_combine_kernel<true><<<grid, 256, 0, st>>>(outputs, n_out, routes, scores, T, k, d, y, err);
  else
    weighted_combine_kernel<false><<<grid, 256, 0, st>>>(outputs, n_out, routes, scores, T, k, d, y, err);
  return cudaGetLastError();
}

}  // namespace vx
