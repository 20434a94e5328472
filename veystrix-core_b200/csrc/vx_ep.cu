// Expert-parallel exchange over NVLink peer memory (B200, one process per
// GPU, every rank's exchange buffer mapped into every other rank).
//
// A step for T tokens on each of P ranks (the same T everywhere):
//   dispatch  rank r stores, into the buffer of every rank p that owns one of
//             token t's experts, the row x[t] (4 KiB at d=2048) at block r,
//             and into every rank the slot ids local to p (-1: elsewhere) and
//             the slot weights; the last CTA raises flag_dispatch[r] on all
//             ranks (release at system scope).
//   experts   rank p waits for every flag_dispatch, runs its expert pipeline
//             over the P*T received rows and, in the combine kernel, stores
//             each row's float32 partial sum sum_s bf16(y_s)*w_s straight into
//             block p of the home rank's back buffer, then raises
//             flag_combine[p] there.  The combine is the collective: no
//             staging copy, no library all-to-all.
//   combine   the home rank waits for every flag_combine and adds the
//             partials in rank order (absent ones as +0.0), rounds once to
//             bf16 and adds bf16(sg * shared) - the arithmetic of the
//             single-GPU combine (models/flashnext/metal_runtime.py:315-334).
// Flags carry a step epoch kept in the buffer's header (incremented by the
// combine's last CTA), so a captured CUDA graph replays the step unchanged.
// Every wait is bounded (iteration count and %globaltimer); a wait that runs
// out sets a bit of the caller's error word and the kernel returns.
// Only plain loads and stores cross NVLink: no TMA, no multicast.
#include <cuda_runtime.h>
#include <stdint.h>

#include "vx_common.cuh"
#include "vx_launch.h"

namespace vx {

namespace {

constexpr int kHdrFlagDispatch = 0;   // u32 [8]
constexpr int kHdrFlagCombine = 8;    // u32 [8]
constexpr int kHdrEpoch = 16;         // u32
constexpr int kHdrTicket = 17;        // u32 [3]: dispatch, send, combine
constexpr uint32_t kWaitIters = 1u << 28;

VX_DEVICE uint32_t* header(unsigned char* buf) { return reinterpret_cast<uint32_t*>(buf); }

VX_DEVICE uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

VX_DEVICE uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

VX_DEVICE void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Waits until *flag has reached epoch e (modulo 2^32); false when the wait
// ran out (limit_ns, or 2^28 polls).
VX_DEVICE bool wait_epoch(const uint32_t* flag, uint32_t e, uint64_t limit_ns) {
  const uint64_t t0 = globaltimer();
  for (uint32_t it = 0; it < kWaitIters; ++it) {
    if (int32_t(ld_acquire_sys(flag) - e) >= 0) return true;
    if ((it & 255u) == 255u && globaltimer() - t0 > limit_ns) return false;
    __nanosleep(32);
  }
  return false;
}

VX_DEVICE uint32_t step_epoch(const EpArgs& a) {
  return *reinterpret_cast<volatile uint32_t*>(header(a.buf[a.rank]) + kHdrEpoch) + 1u;
}

// Publishes this launch's peer stores: the CTA barrier orders its threads'
// stores before thread 0's acquire-release ticket add at system scope (the
// release of this CTA's stores); the CTA that arrives last has acquired every
// other CTA's release and raises flag[slot + rank] = e on every rank with a
// release store (cumulative, so it covers all of them), then re-arms the
// ticket.  No full fence: those cost microseconds each.
VX_DEVICE void signal_all(const EpArgs& a, int ticket, int slot, uint32_t e) {
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t* tk = header(a.buf[a.rank]) + kHdrTicket + ticket;
    uint32_t n;
    asm volatile("atom.acq_rel.sys.global.add.u32 %0, [%1], 1;" : "=r"(n) : "l"(tk) : "memory");
    if (n == gridDim.x * gridDim.y - 1) {
      for (int p = 0; p < a.P; ++p) st_release_sys(header(a.buf[p]) + slot + a.rank, e);
      atomicExch(tk, 0u);
    }
  }
}

// One CTA per (token, destination rank).
__global__ void __launch_bounds__(256) ep_dispatch_kernel(EpArgs a, const uint16_t* __restrict__ x,
                                                          const int32_t* __restrict__ inds,
                                                          const uint16_t* __restrict__ wts) {
  chain_begin();
  const uint32_t e = step_epoch(a);
  const int t = blockIdx.x / a.P, p = blockIdx.x % a.P;
  unsigned char* dst = a.buf[p];
  const int64_t row = int64_t(a.rank) * a.T + t;
  __shared__ int any;
  if (threadIdx.x == 0) any = 0;
  __syncthreads();
  if (threadIdx.x < a.k) {
    const int s = threadIdx.x;
    const int g = inds[int64_t(t) * a.k + s];
    const int lo = p * a.El;
    const int local = (g >= lo && g < lo + a.El) ? g - lo : -1;
    reinterpret_cast<int32_t*>(dst + a.off_ids)[row * a.k + s] = local;
    reinterpret_cast<uint16_t*>(dst + a.off_w)[row * a.k + s] = wts[int64_t(t) * a.k + s];
    if (local >= 0) any = 1;
  }
  __syncthreads();
  if (any) {
    const int4* src = reinterpret_cast<const int4*>(x + int64_t(t) * a.d);
    int4* out = reinterpret_cast<int4*>(dst + a.off_x) + row * (a.d / 8);
    for (int i = threadIdx.x; i < a.d / 8; i += blockDim.x) out[i] = src[i];
  }
  signal_all(a, 0, kHdrFlagDispatch, e);
}

__global__ void ep_wait_dispatch_kernel(EpArgs a) {
  chain_begin();
  const uint32_t e = step_epoch(a);
  if (threadIdx.x < a.P &&
      !wait_epoch(header(a.buf[a.rank]) + kHdrFlagDispatch + threadIdx.x, e, a.wait_ns) && a.err)
    atomicOr(a.err, 1);
}

// One CTA per received row i = r*T + t: the float32 sum over its present
// slots of bf16(y_s)*w_s (slot order, separate multiply and add roundings, as
// combine_partial_kernel), stored into block `rank` of rank r's back buffer.
// Rows with no slot here send nothing.
__global__ void __launch_bounds__(256) ep_send_kernel(EpArgs a, const uint16_t* __restrict__ yd,
                                                      int64_t ldy, const int32_t* __restrict__ inverse) {
  chain_begin();
  const uint32_t e = step_epoch(a);
  const int i = blockIdx.x;
  const int r = i / a.T, t = i % a.T;
  const int32_t* inv = inverse + int64_t(i) * a.k;
  const uint16_t* w = reinterpret_cast<const uint16_t*>(a.buf[a.rank] + a.off_w) + int64_t(i) * a.k;
  bool any = false;
  for (int s = 0; s < a.k; ++s) any |= inv[s] >= 0;
  if (any) {
    float* out = reinterpret_cast<float*>(a.buf[r] + a.off_back) + (int64_t(a.rank) * a.T + t) * a.d;
    for (int c = threadIdx.x * 4; c < a.d; c += blockDim.x * 4) {
      float v0 = 0.f, v1 = 0.f, v2 = 0.f, v3 = 0.f;
      for (int s = 0; s < a.k; ++s) {
        const int pos = inv[s];
        if (pos < 0) continue;
        const float ws = bf16_to_f32(w[s]);
        const uint2 q = *reinterpret_cast<const uint2*>(yd + int64_t(pos) * ldy + c);
        v0 = __fadd_rn(v0, __fmul_rn(__uint_as_float(q.x << 16), ws));
        v1 = __fadd_rn(v1, __fmul_rn(__uint_as_float(q.x & 0xFFFF0000u), ws));
        v2 = __fadd_rn(v2, __fmul_rn(__uint_as_float(q.y << 16), ws));
        v3 = __fadd_rn(v3, __fmul_rn(__uint_as_float(q.y & 0xFFFF0000u), ws));
      }
      *reinterpret_cast<float4*>(out + c) = make_float4(v0, v1, v2, v3);
    }
  }
  signal_all(a, 1, kHdrFlagCombine, e);
}

VX_DEVICE float add_shared(float routed_bf16, float sgv, const uint16_t* shared, int64_t idx) {
  if (!shared) return routed_bf16;
  const float sy = bf16r(__fmul_rn(sgv, bf16_to_f32(shared[idx])));
  return bf16r(__fadd_rn(routed_bf16, sy));
}

// One CTA per home token.
__global__ void __launch_bounds__(256) ep_combine_kernel(EpArgs a, const int32_t* __restrict__ inds,
                                                         const uint16_t* __restrict__ shared,
                                                         const uint16_t* __restrict__ sg,
                                                         uint16_t* __restrict__ y) {
  chain_begin();
  const uint32_t e = step_epoch(a);
  uint32_t* hdr = header(a.buf[a.rank]);
  if (threadIdx.x < a.P && !wait_epoch(hdr + kHdrFlagCombine + threadIdx.x, e, a.wait_ns) && a.err)
    atomicOr(a.err, 2);
  __syncthreads();
  const int t = blockIdx.x;
  uint32_t mask = 0;
  for (int s = 0; s < a.k; ++s) {
    const int g = inds[int64_t(t) * a.k + s];
    if (g >= 0 && g < a.P * a.El) mask |= 1u << (g / a.El);
  }
  const float* back = reinterpret_cast<const float*>(a.buf[a.rank] + a.off_back);
  const float sgv = shared ? bf16_to_f32(sg[t]) : 0.f;
  for (int c = threadIdx.x * 4; c < a.d; c += blockDim.x * 4) {
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int p = 0; p < a.P; ++p) {
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (mask >> p & 1u)
        v = __ldcg(reinterpret_cast<const float4*>(back + (int64_t(p) * a.T + t) * a.d + c));
      if (p == 0) {
        acc = v;
      } else {
        acc.x = __fadd_rn(acc.x, v.x);
        acc.y = __fadd_rn(acc.y, v.y);
        acc.z = __fadd_rn(acc.z, v.z);
        acc.w = __fadd_rn(acc.w, v.w);
      }
    }
    const int64_t o = int64_t(t) * a.d + c;
    const float r0 = add_shared(bf16r(acc.x), sgv, shared, o + 0);
    const float r1 = add_shared(bf16r(acc.y), sgv, shared, o + 1);
    const float r2 = add_shared(bf16r(acc.z), sgv, shared, o + 2);
    const float r3 = add_shared(bf16r(acc.w), sgv, shared, o + 3);
    uint2 q;
    q.x = uint32_t(f32_to_bf16(r0)) | (uint32_t(f32_to_bf16(r1)) << 16);
    q.y = uint32_t(f32_to_bf16(r2)) | (uint32_t(f32_to_bf16(r3)) << 16);
    *reinterpret_cast<uint2*>(y + o) = q;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    uint32_t* tk = hdr + kHdrTicket + 2;
    if (atomicAdd(tk, 1u) == gridDim.x - 1) {
      atomicExch(hdr + kHdrEpoch, e);
      atomicExch(tk, 0u);
    }
  }
}

}  // namespace

EpLayout ep_layout(int P, int cap, int d, int k) {
  auto al = [](int64_t v) { return (v + 255) & ~int64_t(255); };
  EpLayout L;
  int64_t o = kEpHeaderBytes;
  L.x = o;
  o = al(o + int64_t(P) * cap * d * 2);
  L.ids = o;
  o = al(o + int64_t(P) * cap * k * 4);
  L.w = o;
  o = al(o + int64_t(P) * cap * k * 2);
  L.back = o;
  o = al(o + int64_t(P) * cap * d * 4);
  L.bytes = o;
  return L;
}

cudaError_t launch_ep_dispatch(const EpArgs& a, const uint16_t* x, const int32_t* inds,
                               const uint16_t* wts, cudaStream_t st) {
  if (a.T == 0) return cudaSuccess;
  return launch_chained(ep_dispatch_kernel, dim3(a.T * a.P), dim3(256), 0, st, a, x, inds, wts);
}

cudaError_t launch_ep_wait_dispatch(const EpArgs& a, cudaStream_t st) {
  return launch_chained(ep_wait_dispatch_kernel, dim3(1), dim3(32), 0, st, a);
}

cudaError_t launch_ep_send(const EpArgs& a, const uint16_t* yd, int64_t ldy, const int32_t* inverse,
                           cudaStream_t st) {
  if (a.T == 0) return cudaSuccess;
  return launch_chained(ep_send_kernel, dim3(a.T * a.P), dim3(256), 0, st, a, yd, ldy, inverse);
}

cudaError_t launch_ep_combine(const EpArgs& a, const int32_t* inds, const uint16_t* shared,
                              const uint16_t* sg, uint16_t* y, cudaStream_t st) {
  if (a.T == 0) return cudaSuccess;
  return launch_chained(ep_combine_kernel, dim3(a.T), dim3(256), 0, st, a, inds, shared, sg, y);
}

}  // namespace vx
