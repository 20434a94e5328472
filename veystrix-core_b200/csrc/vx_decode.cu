// The whole MoE block for a few decode tokens in one cooperative launch
// (sm_100a): router logits, softmax/top-k/renorm, the expert sort, the
// routed and shared gate/up projections with SwiGLU, the down projections
// and the score-weighted combine (models/flashnext/metal_runtime.py:799-974,
// the reference's custom executor for <= 8 rows; adaptive_topk.py:54-293).
//
// Why one launch.  At one token the block moves about 24 MB (ten routed
// experts, the shared expert, the router) - 3.6 us at full HBM speed - while
// a chain of separate launches pays a launch gap and a pipeline fill per
// kernel and leaves most SMs idle behind the router's serial tail.  Here
// every SM runs one CTA for the whole block; the CTAs meet at two grid
// barriers (bounded waits on global counters):
//
//   phase R   CTAs [0, L) compute the bf16 logits of 4 experts each (the
//             fused router's mma.sync tile and K slicing, so the logits are
//             the router kernel's bit for bit) before anything else; every
//             CTA then builds the x records, and the other CTAs start on the
//             shared expert, whose gate/up projections need no routing.
//   barrier 1
//   phase G   every CTA reads all logits: warp 1 + t selects token t's top-k
//             and hands the ids to warp 0 (named barrier), which runs the
//             stable expert sort (rank by shuffles over at most 64 routes)
//             and the closed-form task split, while warp 5 + t turns the
//             selected keys into the renormalised weights.  The CTA then
//             takes its byte-balanced slice of the routed gate/up tasks
//             (expert, 16-row tile); its 16 warps split each task's
//             128-input chunks, the CTA adds their partial sums in warp
//             order and applies the bf16 SwiGLU; h goes to global.
//             Down-projection weights stream into shared memory meanwhile.
//   barrier 2
//   phase D   CTA c >= G - n_tiles owns one row tile of the down projection
//             for every expert of the step: it builds the h records of all
//             positions, runs its down tiles from shared memory and combines
//             its rows of y in slot order (float32, no FMA, then the shared
//             part) - the combine needs no third barrier.
//
// Weights come from the tiled resident pool (vx_q4_tile), one record per
// (expert, row tile, 128-input chunk): 2,560 bytes for a gate/up pair of 16
// rows, 1,280 or 2,560 bytes for 16 or 32 down rows.  Lane 0 of a warp
// copies a record into a stage of its ring with one bulk copy (two for the
// 16 owned rows of a down record) onto the stage's mbarrier: at one or a few
// tokens the copies are latency-bound, and the copy engine keeps more
// of them in flight per SM than per-lane 16-byte copies (C1 34.1 -> 32.5 us).
// The arithmetic of a record is the tiled GEMV's (vx_gemv_tiled.cu):
// nibbles to bf16 128+q by one lop3, a block-diagonal B operand on mma.sync
// so each MMA yields per-group sums, and MLX's qmv formula
// scale*sum(qx) + bias*sum(x) per group in float32.
//
// No cluster multicast; every copy lands in the issuing CTA's own shared
// memory.  Every wait is bounded: a grid barrier gives up after wait_ns
// (error bit 0x400), an mbarrier after kSpinLimit polls (0x100); the kernel
// then waits (bounded) for its own copies in flight and returns.
#include <type_traits>

#include "vx_async.cuh"
#include "vx_common.cuh"
#include "vx_launch.h"
#include "vx_topk.cuh"

namespace vx {

constexpr int kDecThreads = 512;
constexpr int kDecWarps = kDecThreads / 32;
constexpr int kDecStage = 2560;         // one pool record (largest: gate/up pair, 32 down rows)
constexpr int kDecLogitRows = 4;        // experts per logit CTA
constexpr int kDecMaxRoutes = 64;       // T*k for the one-warp sort
static_assert(kDecWarps >= 5 + kDecodeMaxT, "routing warps: 0 plans, 1..T select, 5..4+T weigh");
// gate/up partial sums: [task][warp][projection][row 16][token T] float in a
// region of kDecPartBytes, so a batch holds kDecPartBytes / (1 KB * T) tasks
constexpr int kDecPartBytes = 16384;

// ---------------------------------------------------------------------------
// Shared-memory layout (the host computes the same numbers to size the launch)
// ---------------------------------------------------------------------------

struct DecLayout {
  int nch_d, nch_h, Pp, tile_rows, nch_s;
  int off_x, off_h, off_y, off_sd, off_part, off_tab, off_bar, off_ring;
  int ring_stages, total;
};

VX_HOST_DEVICE inline int dec_align(int v, int a) { return (v + a - 1) / a * a; }

VX_HOST_DEVICE inline DecLayout dec_layout(int T, int d, int k, int I, int Is, int dn_mt, int smem_cap) {
  DecLayout L;
  L.nch_d = d / 128;
  L.nch_h = (I > Is ? I : Is) / 128;
  L.nch_s = Is / 128;
  L.Pp = T * k + (Is > 0 ? T : 0);
  L.tile_rows = 16;                                     // rows of y a down owner computes
  int off = 0;
  L.off_x = off;                                        // x records [nch_d][T][320]
  off += dec_align(L.nch_d * T * kActRecord, 128);
  L.off_h = off;                                        // h records [nch_h][Pp][320]
  int hbytes = L.nch_h * L.Pp * kActRecord;
  const int logit_scratch = kDecWarps * 32 * 4 * 4;     // phase R: router K-slice partials
  if (hbytes < logit_scratch) hbytes = logit_scratch;
  off += dec_align(hbytes, 128);
  L.off_y = off;                                        // down outputs [Pp][tile_rows] bf16
  off += dec_align(L.Pp * L.tile_rows * 2, 128);
  L.off_sd = off;                                       // the shared expert's down records
  off += (Is > 0 ? L.nch_s * 1280 : 0);
  L.off_part = off;                                     // gate/up partial sums
  off += kDecPartBytes;
  L.off_tab = off;                                      // routing tables
  off += dec_align(kDecMaxRoutes * 4 * 2 + kDecMaxRoutes * 2 + (kDecMaxRoutes + 16) * 4 +
                       (kDecMaxRoutes + 2) * 4 * 3 + 64 * 4 + kDecMaxRoutes * 4,
                   128);
  L.off_bar = off;                                      // ring mbarriers + the shared-down one
  const int avail = smem_cap - off;
  int stages = (avail - 256) / (kDecStage + 8);
  stages = stages / kDecWarps * kDecWarps;
  L.ring_stages = stages;
  off += dec_align((stages + 1) * 8, 128);
  L.off_ring = off;
  off += stages * kDecStage;
  L.total = off;
  return L;
}

// Routing tables inside off_tab.
struct DecTab {
  int32_t* inds;      // [T*k] routed expert ids (flat t*k+s)
  int32_t* posof;     // [T*k] sorted position of flat index (-1: dropped)
  uint16_t* wts;      // [T*k] renormalised weights (bf16 bits)
  int32_t* tok;       // [Pp] token of each sorted position
  int32_t* ex;        // [U+1] expert of slot u (E: the shared expert)
  int32_t* p0;        // [U+1] first position of slot u
  int32_t* cnt;       // [U+1] positions of slot u
  int32_t* plan;      // U, first task, tasks, abort flag
  uint32_t* keys;     // [T*k] selected keys (top-k to the weights warps)
};

VX_DEVICE DecTab dec_tab(unsigned char* base) {
  DecTab t;
  t.inds = reinterpret_cast<int32_t*>(base);
  t.posof = t.inds + kDecMaxRoutes;
  t.wts = reinterpret_cast<uint16_t*>(t.posof + kDecMaxRoutes);
  t.tok = reinterpret_cast<int32_t*>(t.wts + kDecMaxRoutes);
  t.ex = t.tok + kDecMaxRoutes + 16;
  t.p0 = t.ex + kDecMaxRoutes + 2;
  t.cnt = t.p0 + kDecMaxRoutes + 2;
  t.plan = t.cnt + kDecMaxRoutes + 2;
  t.keys = reinterpret_cast<uint32_t*>(t.plan + 64);
  return t;
}

enum { kPlanU = 0, kPlanFirst = 1, kPlanNr = 2, kPlanAbort = 3 };

// ---------------------------------------------------------------------------
// grid barrier: arrive (release) and bounded wait (acquire) on a counter that
// is zero at launch
// ---------------------------------------------------------------------------

VX_DEVICE uint64_t gtimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

VX_DEVICE void grid_arrive(uint32_t* ctr) {
  asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(ctr) : "memory");
}

VX_DEVICE bool grid_wait(const uint32_t* ctr, uint32_t target, uint64_t limit_ns) {
  const uint64_t t0 = gtimer();
  for (uint32_t i = 0; i < (1u << 26); ++i) {
    uint32_t v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(ctr) : "memory");
    if (v >= target) return true;
    if ((i & 15u) == 15u && gtimer() - t0 > limit_ns) return false;
  }
  return false;
}

// ---------------------------------------------------------------------------
// activation records (B operand of the record MMAs): one thread per 8-input
// block, the four blocks of a quant group on adjacent lanes; the group sum is
// left-to-right over 8 inputs, then (s0+s1)+(s2+s3), as act_records_kernel.
// ---------------------------------------------------------------------------

VX_DEVICE void put_record_block(unsigned char* rec, int blk, uint4 v, bool live) {
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
  const int c = (blk >> 2) & 3, ib = blk & 3;
  uint4 o;
  o.x = prmt(v.x, v.z, 0x5410);
  o.y = prmt(v.x, v.z, 0x7632);
  o.z = prmt(v.y, v.w, 0x5410);
  o.w = prmt(v.y, v.w, 0x7632);
  *reinterpret_cast<uint4*>(rec + (ib * 4 + c) * 16) = o;
  if (ib == 0) *reinterpret_cast<float*>(rec + kActXsum + c * 4) = s;
}

// ---------------------------------------------------------------------------
// one record on the tensor pipe: NM 16-row blocks (gate and up of a pair, or
// the m-tiles of a down record) against NQ B operands of two tokens each
// ---------------------------------------------------------------------------

template <int NQ, int NM>
VX_DEVICE void rec_mma(uint32_t st, uint32_t brec, const uint32_t (&tokoff)[4], int cnt, uint32_t zaddr,
                       float (&acc)[NM][2][2]) {
  const int lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
  const bool blane = (g & 3) == c;
  const int tb = g >> 2, ts = c >> 1;
  uint32_t bq[NQ][16];
  float xs[NQ][2];
#pragma unroll
  for (int q = 0; q < NQ; ++q) {
    const int jb = 2 * q + tb, js = 2 * q + ts;
    const bool live = blane && jb < cnt;
    const uint32_t base = live ? brec + tokoff[jb] + c * 16 : zaddr;
    const uint32_t step = live ? 64 : 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint4 v = lds128(base + i * step);
      bq[q][4 * i + 0] = v.x;
      bq[q][4 * i + 1] = v.y;
      bq[q][4 * i + 2] = v.z;
      bq[q][4 * i + 3] = v.w;
    }
    const uint2 v = lds64(js < cnt ? brec + tokoff[js] + kActXsum + (c & 1) * 8 : zaddr);
    xs[q][0] = __uint_as_float(v.x);
    xs[q][1] = __uint_as_float(v.y);
  }
  // The MMAs of every 16-row block first, blocks interleaved, so that 2 x NM
  // (for a single block 4) independent accumulator chains are in flight: a
  // record on one warp is bound by the dependent MMA latency.  The chains
  // are added in a fixed order at the end.
  constexpr int NC = NM == 1 ? 4 : 2;   // chains per block
  uint32_t ag[NM][4], a8[NM][4];
#pragma unroll
  for (int pm = 0; pm < NM; ++pm) {
    const uint32_t wrow = st + pm * 1024 + lane * 16;
    const uint4 wg = lds128(wrow), w8 = lds128(wrow + 512);
    ag[pm][0] = wg.x, ag[pm][1] = wg.y, ag[pm][2] = wg.z, ag[pm][3] = wg.w;
    a8[pm][0] = w8.x, a8[pm][1] = w8.y, a8[pm][2] = w8.z, a8[pm][3] = w8.w;
  }
  float dc[NM][NC][NQ][4];
#pragma unroll
  for (int pm = 0; pm < NM; ++pm)
#pragma unroll
    for (int cc = 0; cc < NC; ++cc)
#pragma unroll
      for (int q = 0; q < NQ; ++q)
#pragma unroll
        for (int i = 0; i < 4; ++i) dc[pm][cc][q][i] = 0.f;
#pragma unroll
  for (int wi = 0; wi < 4; ++wi) {
    const int mm = 2 * wi;
    const int cf = NC == 4 ? 2 * (wi & 1) : 0;   // chain of the low nibble pairs; +1: the high ones
#pragma unroll
    for (int pm = 0; pm < NM; ++pm) {
      const uint32_t f0 = nib_pair128(ag[pm][wi]), f1 = nib_pair128(a8[pm][wi]);
      const uint32_t f2 = nib_pair128(ag[pm][wi] >> 4), f3 = nib_pair128(a8[pm][wi] >> 4);
      const uint32_t h0 = nib_pair128(ag[pm][wi] >> 8), h1 = nib_pair128(a8[pm][wi] >> 8);
      const uint32_t h2 = nib_pair128(ag[pm][wi] >> 12), h3 = nib_pair128(a8[pm][wi] >> 12);
#pragma unroll
      for (int q = 0; q < NQ; ++q) {
        mma16816(dc[pm][cf][q], f0, f1, f2, f3, bq[q][2 * mm], bq[q][2 * mm + 1]);
        mma16816(dc[pm][cf + 1][q], h0, h1, h2, h3, bq[q][2 * mm + 2], bq[q][2 * mm + 3]);
      }
    }
  }
#pragma unroll
  for (int pm = 0; pm < NM; ++pm) {
    float d[NQ][4];
#pragma unroll
    for (int q = 0; q < NQ; ++q)
#pragma unroll
      for (int i = 0; i < 4; ++i)
        d[q][i] = NC == 4 ? (dc[pm][0][q][i] + dc[pm][2][q][i]) + (dc[pm][1][q][i] + dc[pm][3][q][i])
                          : dc[pm][0][q][i] + dc[pm][1][q][i];
    const uint4 sb = lds128(st + NM * 1024 + pm * 256 + (g * 2 + (c & 1)) * 16);
    const uint32_t sw[4] = {sb.x, sb.y, sb.z, sb.w};
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const float s0 = __uint_as_float(sw[2 * h] << 16);
      const float s1 = __uint_as_float(sw[2 * h] & 0xFFFF0000u);
      const float b0 = __uint_as_float(sw[2 * h + 1] << 16);
      const float b1 = __uint_as_float(sw[2 * h + 1] & 0xFFFF0000u);
      const float c0 = fmaf(-128.f, s0, b0);   // the lop3 operands carry q + 128
      const float c1 = fmaf(-128.f, s1, b1);
#pragma unroll
      for (int q = 0; q < NQ; ++q) {
        float v = acc[pm][q][h];
        v = fmaf(s0, d[q][2 * h], v);
        v = fmaf(c0, xs[q][0], v);
        v = fmaf(s1, d[q][2 * h + 1], v);
        v = fmaf(c1, xs[q][1], v);
        acc[pm][q][h] = v;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// per-warp stream of records: [shared gate/up chunks][routed gate/up chunks]
// [routed down records], each warp taking chunks ch = w, w + 8, ... of every
// gate/up task and the down jobs (experts) dj = w, w + 8, ...
// ---------------------------------------------------------------------------

struct DecPlan {
  int T, k, E, d, G, L, n_dt;   // n_dt: 16-row tiles of y, one per down owner
  int P, nch_d, nch_i, rbg, dn_mt;
  int ns;              // shared gate/up tasks of this CTA
  int U, first, nr;    // routed: distinct experts, first task, tasks of this CTA (after routing)
  int td;              // 16-row tile of y this CTA owns, or -1
  bool routed;         // routing known
};

struct GuTask {
  int u, rb;           // slot (-1: the shared expert), 16-row tile
};

VX_DEVICE GuTask shared_task(const DecPlan& pl, int j) {
  // the CTA's j-th shared task: global shared task id (c - L) + j*(G - L)
  const int span = pl.G - pl.L;
  return {-1, int(blockIdx.x) - pl.L + j * span};
}

VX_DEVICE GuTask routed_task(const DecPlan& pl, int j) {
  const int r = pl.first + j;
  const int u = r / pl.rbg;
  return {u, r - u * pl.rbg};
}

struct DecCursor {
  int ph;   // 0 shared gate/up, 1 routed gate/up, 2 routed down, 3 end
  int j;    // task / job index within the phase
  int ch;   // chunk
};

// First valid record at or after the cursor; false when the stream is
// exhausted or its next phase needs the routing that is not known yet.
VX_DEVICE bool dec_seek(const DecPlan& pl, int warp, DecCursor& cu) {
  for (;;) {
    if (cu.ph == 0) {
      if (cu.j < pl.ns && cu.ch < pl.nch_d) return true;
      if (cu.j < pl.ns) {
        ++cu.j;
        cu.ch = warp;
        continue;
      }
      cu.ph = 1;
      cu.j = 0;
      cu.ch = warp;
    }
    if (cu.ph == 1) {
      if (!pl.routed) return false;
      if (cu.j < pl.nr && cu.ch < pl.nch_d) return true;
      if (cu.j < pl.nr) {
        ++cu.j;
        cu.ch = warp;
        continue;
      }
      cu.ph = 2;
      cu.j = warp;
      cu.ch = 0;
    }
    if (cu.ph == 2) {
      if (pl.td >= 0 && cu.j < pl.U) {
        if (cu.ch < pl.nch_i) return true;
        cu.j += kDecWarps;
        cu.ch = 0;
        continue;
      }
      cu.ph = 3;
    }
    return false;
  }
}

VX_DEVICE void dec_advance(DecCursor& cu) {
  if (cu.ph == 2)
    ++cu.ch;
  else
    cu.ch += kDecWarps;
}

// Per-warp ring state.
struct DecRing {
  uint32_t base, bar0;   // first stage / mbarrier of this warp
  int R;                 // stages
  int issued, used;      // records issued / consumed
  DecCursor cur;         // next record to issue
  bool timed_out;
};

// Issues records into free stages: lane 0 arms the stage's mbarrier (count
// 1) with the record's bytes and bulk-copies it (after a proxy fence: the
// stage was last read through the generic proxy).
VX_DEVICE void ring_fill(const DecodeArgs& a, const DecPlan& pl, const DecTab& tb, DecRing& rg, int warp,
                         uint64_t pol) {
  const int lane = threadIdx.x & 31;
  while (rg.issued - rg.used < rg.R && dec_seek(pl, warp, rg.cur)) {
    const int s = rg.issued % rg.R;
    const uint32_t dst = rg.base + s * kDecStage;
    if (rg.cur.ph <= 1) {
      // a whole gate/up record: both projections of a 16-row tile
      const GuTask t = rg.cur.ph == 0 ? shared_task(pl, rg.cur.j) : routed_task(pl, rg.cur.j);
      const unsigned char* rec =
          t.u < 0 ? a.gu_rec_s : a.gu_rec + routed_record(a.slot_of, a.slots, tb.ex[t.u]) * a.gu_stride;
      const unsigned char* src = rec + (int64_t(t.rb) * pl.nch_d + rg.cur.ch) * 2560;
      if (lane == 0) {
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        mbar_expect(rg.bar0 + 8 * s, 2560);
        bulk_load(dst, src, 2560, rg.bar0 + 8 * s, pol);
      }
    } else {
      // the 16 owned rows of a down record (record tile td / dn_mt, m-tile
      // td % dn_mt): their packed words, then their scales and biases
      const int m = pl.td % pl.dn_mt;
      const unsigned char* rec = a.dn_rec + routed_record(a.slot_of, a.slots, tb.ex[rg.cur.j]) * a.dn_stride +
                                 (int64_t(pl.td / pl.dn_mt) * pl.nch_i + rg.cur.ch) * (pl.dn_mt * 1280);
      if (lane == 0) {
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        mbar_expect(rg.bar0 + 8 * s, 1280);
        bulk_load(dst, rec + m * 1024, 1024, rg.bar0 + 8 * s, pol);
        bulk_load(dst + 1024, rec + pl.dn_mt * 1024 + m * 256, 256, rg.bar0 + 8 * s, pol);
      }
    }
    ++rg.issued;
    dec_advance(rg.cur);
  }
}

// Waits for the next record in the ring and returns its stage address.
VX_DEVICE uint32_t ring_take(DecRing& rg) {
  const int s = rg.used % rg.R;
  const uint32_t parity = uint32_t(rg.used / rg.R) & 1u;
  if (!mbar_wait(rg.bar0 + 8 * s, parity)) rg.timed_out = true;
  return rg.base + s * kDecStage;
}

VX_DEVICE void ring_release(DecRing& rg) {
  __syncwarp();   // every lane has read the stage before any lane refills it
  ++rg.used;
}

// Before an early return: wait (bounded) for this warp's copies in flight.
VX_DEVICE void ring_drain(DecRing& rg) {
  while (rg.used < rg.issued) {
    ring_take(rg);
    ring_release(rg);
  }
}

VX_DEVICE void mbar_init_count(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

// ---------------------------------------------------------------------------
// the kernel
// ---------------------------------------------------------------------------

template <int PER, int DNMT>
__global__ void __launch_bounds__(kDecThreads, 1) decode_kernel(const __grid_constant__ DecodeArgs a) {
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ __align__(16) uint32_t zero16[4];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int T = a.T, k = a.k, E = a.E, d = a.d;
  const int G = gridDim.x;
  const DecLayout lay = dec_layout(T, d, k, a.I, a.Is, DNMT, a.smem_bytes);
  DecTab tb = dec_tab(smem + lay.off_tab);
  const uint32_t zaddr = smem_u32(zero16);
  const uint64_t pol = policy_evict_first();

  DecPlan pl;
  pl.T = T;
  pl.k = k;
  pl.E = E;
  pl.d = d;
  pl.G = G;
  pl.L = (E + kDecLogitRows - 1) / kDecLogitRows;
  pl.n_dt = (d + 15) / 16;
  pl.P = T * k;
  pl.nch_d = lay.nch_d;
  pl.nch_i = a.I / 128;
  pl.rbg = a.I / 16;
  pl.dn_mt = DNMT;
  const int ns_total = a.Is / 16;   // shared gate/up tasks (16-row tiles)
  {
    const int base = int(blockIdx.x) - pl.L, span = G - pl.L;
    pl.ns = (base < 0 || base >= ns_total) ? 0 : (ns_total - base + span - 1) / span;
  }
  pl.U = 0;
  pl.first = 0;
  pl.nr = 0;
  pl.td = int(blockIdx.x) >= G - pl.n_dt ? int(blockIdx.x) - (G - pl.n_dt) : -1;
  pl.routed = false;
  const bool logit_cta = int(blockIdx.x) < pl.L;

  if (threadIdx.x < 4) zero16[threadIdx.x] = 0u;
  // ---- ring set-up: R stages per warp, one mbarrier (32 arrivals) each
  DecRing rg;
  rg.R = lay.ring_stages / kDecWarps;
  rg.base = smem_u32(smem + lay.off_ring) + warp * rg.R * kDecStage;
  rg.bar0 = smem_u32(smem + lay.off_bar) + warp * rg.R * 8;
  rg.issued = rg.used = 0;
  rg.cur = {0, 0, warp};
  rg.timed_out = false;
  if (lane == 0)
    for (int s = 0; s < rg.R; ++s) mbar_init_count(rg.bar0 + 8 * s, 1);
  const uint32_t sd_bar = smem_u32(smem + lay.off_bar) + lay.ring_stages * 8;
  const bool sd_owner = pl.td >= 0 && a.Is > 0;
  if (threadIdx.x == 0) {
    tb.plan[kPlanAbort] = 0;
    if (sd_owner) mbar_init(sd_bar);
  }
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  __syncthreads();

  // ---- routing-independent copies: shared gate/up records, and the shared
  // expert's down records of a down owner (their own region, bulk copies)
  ring_fill(a, pl, tb, rg, warp, pol);
  if (sd_owner && threadIdx.x == 0) {
    // the shared expert's owned rows, one 1,280-byte unit per chunk
    const int m = pl.td % DNMT;
    mbar_expect(sd_bar, uint32_t(lay.nch_s * 1280));
    for (int ch = 0; ch < lay.nch_s; ++ch) {
      const unsigned char* rec = a.dn_rec_s + (int64_t(pl.td / DNMT) * lay.nch_s + ch) * (DNMT * 1280);
      const uint32_t dst = smem_u32(smem + lay.off_sd) + ch * 1280;
      bulk_load(dst, rec + m * 1024, 1024, sd_bar, pol);
      bulk_load(dst + 1024, rec + DNMT * 1024 + m * 256, 256, sd_bar, pol);
    }
  }

  // ---- phase R: logits (CTAs [0, L)), shared gate (CTA L)
  if (logit_cta) {
    // the fused router's 16 x 8 tile with rows g < 4 only (the other rows
    // zero; an MMA output element depends on its own row alone): the same K
    // slices per warp (of the router's 8) and the same slice-order
    // reduction, so each logit equals router_fused_kernel's
    float* red = reinterpret_cast<float*>(smem + lay.off_h);   // [warps][32][4]
    const int g = lane >> 2, c = lane & 3;
    const int ea = int(blockIdx.x) * kDecLogitRows + g, tx = g;
    const bool row_live = g < kDecLogitRows && ea < E;
    const uint16_t* ra = a.router_w + int64_t(row_live ? ea : 0) * d;
    const uint16_t* rx = a.x + int64_t(tx < T ? tx : 0) * d;
    constexpr int kSlices = 8;   // the fused router's K slices (one per warp there)
    const int steps = d / 32;
    const int per = (steps + kSlices - 1) / kSlices;
    const int s0 = warp < kSlices ? warp * per : steps, s1 = min(steps, s0 + per);
    float dd[4] = {0.f, 0.f, 0.f, 0.f};
    constexpr int kBatch = 8;
    const uint4 zero = make_uint4(0, 0, 0, 0);
    for (int sb = s0; sb < s1; sb += kBatch) {
      uint4 wa[kBatch], xb[kBatch];
#pragma unroll
      for (int i = 0; i < kBatch; ++i) {
        const int s = sb + i;
        const int kk = s * 32 + c * 8;
        wa[i] = (s < s1 && row_live) ? ldg_keep(ra + kk) : zero;
        xb[i] = (s < s1 && tx < T) ? __ldg(reinterpret_cast<const uint4*>(rx + kk)) : zero;
      }
#pragma unroll
      for (int i = 0; i < kBatch; ++i) {
        if (sb + i < s1) {
          mma16816(dd, wa[i].x, 0u, wa[i].y, 0u, xb[i].x, xb[i].y);
          mma16816(dd, wa[i].z, 0u, wa[i].w, 0u, xb[i].z, xb[i].w);
        }
      }
    }
    if (warp < kSlices)
#pragma unroll
      for (int i = 0; i < 4; ++i) red[(warp * 32 + lane) * 4 + i] = dd[i];
    __syncthreads();
    if (warp == 0) {
      float v[2] = {0.f, 0.f};
      for (int w = 0; w < kSlices; ++w)
#pragma unroll
        for (int i = 0; i < 2; ++i) v[i] += red[(w * 32 + lane) * 4 + i];
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int t = 2 * c + i;
        if (row_live && t < T) {
          float l = bf16r(v[i]);
          if (a.router_bias) l = bf16r(__fadd_rn(l, bf16_to_f32(a.router_bias[ea])));
          a.logits[int64_t(t) * E + ea] = f32_to_bf16(l);
        }
      }
    }
  } else if (int(blockIdx.x) == pl.L && a.seg.w) {
    // sigmoid(shared_expert_gate(x)): warp t -> token t (the router's code)
    const int t = warp;
    if (t < T) {
      const int Gq = d / 32;
      const uint16_t* xr = a.x + int64_t(t) * d;
      float acc = 0.f;
      for (int gq = lane; gq < Gq; gq += 32) {
        const uint4 w = __ldg(reinterpret_cast<const uint4*>(a.seg.w) + gq);
        const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
        float q = 0.f, xs = 0.f;
#pragma unroll
        for (int cc = 0; cc < 4; ++cc) {
          const uint4 xv = __ldg(reinterpret_cast<const uint4*>(xr + gq * 32 + cc * 8));
          const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
          for (int n = 0; n < 8; ++n) {
            const float v = __uint_as_float((n & 1) ? (xw[n >> 1] & 0xFFFF0000u) : (xw[n >> 1] << 16));
            q = fmaf(float(nibble(ws[cc], n)), v, q);
            xs += v;
          }
        }
        acc += fmaf(bf16_to_f32(a.seg.scales[gq]), q, bf16_to_f32(a.seg.biases[gq]) * xs);
      }
      acc = warp_sum<32>(acc);
      if (lane == 0) a.sg[t] = f32_to_bf16(sigmoid_bf16(bf16r(acc)));
    }
  }
  __syncthreads();   // logits / sg stored
  if (threadIdx.x == 0) grid_arrive(a.sync + 0);

  // ---- x activation records (every CTA, all tokens), after the logits so
  // that the first barrier waits on the router alone
  {
    const int n = T * pl.nch_d * 16;   // whole warps run the loop (shuffles inside)
    for (int i = threadIdx.x; i < ((n + 31) & ~31); i += kDecThreads) {
      const bool live = i < n;
      const int t = live ? i / (pl.nch_d * 16) : 0, r = live ? i - t * pl.nch_d * 16 : 0;
      const int ch = r >> 4, blk = r & 15;
      const uint4 v = live ? *reinterpret_cast<const uint4*>(a.x + int64_t(t) * d + ch * 128 + blk * 8)
                           : make_uint4(0, 0, 0, 0);
      put_record_block(smem + lay.off_x + (ch * T + t) * kActRecord, blk, v, live);
    }
  }
  if (threadIdx.x < T) tb.tok[pl.P + threadIdx.x] = threadIdx.x;   // shared positions P + t
  __syncthreads();   // x records built

  float* part = reinterpret_cast<float*>(smem + lay.off_part);

  // Runs `n` gate/up tasks (phase ph) in batches of `batch`: every warp
  // its chunks of each task into its partial sums, then the CTA adds the
  // warps' partials in warp order, rounds g and u to bf16, applies the bf16
  // SwiGLU and stores h to global.
  const int pw_floats = 2 * 16 * T;                         // one (task, warp)
  const int batch = kDecPartBytes / (kDecWarps * pw_floats * 4);
  auto run_gu = [&](int ph, int n) {
    for (int b0 = 0; b0 < n; b0 += batch) {
      const int nb = min(batch, n - b0);
      for (int jb = 0; jb < nb; ++jb) {
        const GuTask t = ph == 0 ? shared_task(pl, b0 + jb) : routed_task(pl, b0 + jb);
        const int p0 = t.u < 0 ? pl.P : tb.p0[t.u];
        const int cnt = t.u < 0 ? T : tb.cnt[t.u];
        uint32_t tokoff[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) tokoff[q] = q < cnt ? uint32_t(tb.tok[p0 + q]) * kActRecord : 0u;
        float acc[2][2][2] = {};
        for (int ch = warp; ch < pl.nch_d; ch += kDecWarps) {
          if (rg.issued - rg.used < rg.R && rg.cur.ph != 3) ring_fill(a, pl, tb, rg, warp, pol);
          const uint32_t st = ring_take(rg);
          const uint32_t brec = smem_u32(smem + lay.off_x) + ch * T * kActRecord;
          if (cnt > 2)
            rec_mma<2, 2>(st, brec, tokoff, cnt, zaddr, acc);
          else
            rec_mma<1, 2>(st, brec, tokoff, cnt, zaddr, acc);
          ring_release(rg);
        }
        float* pw = part + (jb * kDecWarps + warp) * pw_floats;
#pragma unroll
        for (int p = 0; p < 2; ++p)
#pragma unroll
          for (int q = 0; q < 2; ++q)
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const float v = acc[p][q][h] + __shfl_xor_sync(0xFFFFFFFFu, acc[p][q][h], 1);
              const int j = 2 * q + ((lane & 3) >> 1);
              if ((lane & 1) == 0 && j < cnt) pw[(p * 16 + (lane >> 2) + 8 * h) * T + j] = v;
            }
      }
      __syncthreads();
      // reduce: thread -> (task, row, token); h = silu(bf16 g) * bf16 u
      for (int i = threadIdx.x; i < nb * 16 * T; i += kDecThreads) {
        const int jb = i / (16 * T), r = (i / T) & 15, j = i % T;
        const GuTask t = ph == 0 ? shared_task(pl, b0 + jb) : routed_task(pl, b0 + jb);
        const int p0 = t.u < 0 ? pl.P : tb.p0[t.u];
        const int cnt = t.u < 0 ? T : tb.cnt[t.u];
        if (j >= cnt) continue;
        float gv = 0.f, uv = 0.f;
        for (int w = 0; w < kDecWarps; ++w) {
          const float* pw = part + (jb * kDecWarps + w) * pw_floats;
          gv += pw[r * T + j];
          uv += pw[(16 + r) * T + j];
        }
        const float hv = silu_mul_bf16(bf16r(gv), bf16r(uv));
        a.h[int64_t(p0 + j) * a.ldh + t.rb * 16 + r] = f32_to_bf16(hv);
      }
      __syncthreads();
    }
  };

  // ---- shared expert gate/up while the logits are being computed elsewhere
  if (pl.ns > 0) run_gu(0, pl.ns);

  // ---- barrier 1: every logit stored
  if (threadIdx.x == 0) {
    if (!grid_wait(a.sync + 0, uint32_t(G), a.wait_ns)) {
      atomicOr(a.err, 0x400);
      tb.plan[kPlanAbort] = 1;
    }
  }
  __syncthreads();
  if (tb.plan[kPlanAbort]) {
    ring_drain(rg);
    if (sd_owner && threadIdx.x == 0) mbar_wait(sd_bar, 0);
    return;
  }

  // ---- routing: warp 1 + t selects token t's top-k ids (and their keys)
  // and hands them to warp 0 (named barrier 1: the stable expert sort and
  // the task split) and to warp 5 + t (named barrier 2), which meanwhile
  // computed the softmax statistics of token t and now turns the keys into
  // the renormalised weights (needed only by the combine).  Adaptive top-k
  // needs the probabilities to pick the kept slots: the whole of topk_row
  // in warp 1 + t.
  const bool adapt = a.keep_mass > 0.0 && a.keep_mass < 1.0;
  const int nb1 = 32 * (T + 1), nb2 = 64 * T;
  if (warp >= 1 && warp <= T) {
    const int t = warp - 1;
    const uint16_t* lr = a.logits + int64_t(t) * E;
    if (adapt)
      topk_row<PER, true>(lr, E, k, tb.inds + t * k, nullptr, tb.wts + t * k, nullptr, a.keep_mass, a.keep_min);
    else
      topk_select_keys<PER, true>(lr, E, k, tb.inds + t * k, tb.keys + t * k);
    named_arrive(1, nb1);
    named_arrive(2, nb2);
  } else if (warp >= 5 && warp < 5 + T) {
    const int t = warp - 5;
    if (adapt)
      named_sync(2, nb2);
    else
      topk_weights_keys<PER, true>(a.logits + int64_t(t) * E, E, k, tb.keys + t * k, tb.wts + t * k,
                                   [&]() { named_sync(2, nb2); });
  }
  if (warp == 0) {
    named_sync(1, nb1);
    const int P = pl.P;
    // ids outside [0, E) (a selection among NaN logits) are dropped, as the
    // permutation drops them: no position, counted in the error word.  A
    // slot that adaptive top-k dropped (it repeats its token's slot-0 expert
    // with weight 0; top-k ids are otherwise distinct) gets no position
    // either, and is no error: its zero-weighted term is left out of the
    // combine, and an expert never holds more positions than tokens.
    uint32_t kv[2];
    int n_bad = 0;
#pragma unroll
    for (int r = 0; r < 2; ++r) {
      const int i = lane + 32 * r;
      const int e = i < P ? tb.inds[i] : -1;
      const bool ok = i < P && e >= 0 && e < E;
      const bool dropped = ok && adapt && (i % k) != 0 && e == tb.inds[i - i % k];
      n_bad += (i < P && !ok) ? 1 : 0;
      kv[r] = ok && !dropped ? (uint32_t(e) << 6) | uint32_t(i) : 0xFFFFFFFFu;
      if (i < P) tb.posof[i] = -1;
    }
    n_bad = __reduce_add_sync(0xFFFFFFFFu, n_bad);
    if (n_bad && lane == 0 && blockIdx.x == 0) atomicAdd(a.err + 1, n_bad);
    __syncwarp();
    // sorted order by rank: a key's position is the number of keys below it
    // (valid keys are distinct: the flat index is part of the key); the
    // sorted keys go through shared memory (the plan region is free here)
    {
      // (keys past P are 0xFFFFFFFF and rank below nothing: only the P
      // routed keys are visited)
      int ra = 0, rb = 0;
      const int n0 = P < 32 ? P : 32, n1 = P > 32 ? P - 32 : 0;
#pragma unroll 4
      for (int j = 0; j < n0; ++j) {
        const uint32_t xa = __shfl_sync(0xFFFFFFFFu, kv[0], j);
        ra += xa < kv[0];
        rb += xa < kv[1];
      }
#pragma unroll 4
      for (int j = 0; j < n1; ++j) {
        const uint32_t xb = __shfl_sync(0xFFFFFFFFu, kv[1], j);
        ra += xb < kv[0];
        rb += xb < kv[1];
      }
      uint32_t* skey = reinterpret_cast<uint32_t*>(part);
      skey[lane] = skey[lane + 32] = 0xFFFFFFFFu;
      __syncwarp();
      if (kv[0] != 0xFFFFFFFFu) skey[ra] = kv[0];
      if (kv[1] != 0xFFFFFFFFu) skey[rb] = kv[1];
      __syncwarp();
      kv[0] = skey[lane];
      kv[1] = skey[lane + 32];
    }
    const uint32_t e0 = kv[0] >> 6, e1 = kv[1] >> 6;
    const uint32_t prev0 = __shfl_up_sync(0xFFFFFFFFu, e0, 1);
    uint32_t prev1 = __shfl_up_sync(0xFFFFFFFFu, e1, 1);
    const uint32_t last0 = __shfl_sync(0xFFFFFFFFu, e0, 31);
    if (lane == 0) prev1 = last0;
    const bool v0 = kv[0] != 0xFFFFFFFFu, v1 = kv[1] != 0xFFFFFFFFu;
    const int Pv = __popc(__ballot_sync(0xFFFFFFFFu, v0)) + __popc(__ballot_sync(0xFFFFFFFFu, v1));
    const bool h0 = v0 && (lane == 0 || e0 != prev0);
    const bool h1 = v1 && e1 != prev1;
    const uint32_t b0 = __ballot_sync(0xFFFFFFFFu, h0), b1 = __ballot_sync(0xFFFFFFFFu, h1);
    const uint32_t lt = (1u << lane) - 1u;
    const int U = __popc(b0) + __popc(b1);
    if (v0) {
      const int f = int(kv[0] & 63u);
      tb.posof[f] = lane;
      tb.tok[lane] = f / k;
    }
    if (v1) {
      const int f = int(kv[1] & 63u);
      tb.posof[f] = lane + 32;
      tb.tok[lane + 32] = f / k;
    }
    if (h0) {
      const int u = __popc(b0 & lt);
      tb.ex[u] = int(e0);
      tb.p0[u] = lane;
    }
    if (h1) {
      const int u = __popc(b0) + __popc(b1 & lt);
      tb.ex[u] = int(e1);
      tb.p0[u] = lane + 32;
    }
    if (lane == 0) tb.plan[kPlanU] = U;
    __syncwarp();
    for (int u = lane; u < U; u += 32) tb.cnt[u] = (u + 1 < U ? tb.p0[u + 1] : Pv) - tb.p0[u];

    // ---- byte-balanced split of the routed gate/up tasks over the CTAs (in
    // units of 256 bytes) for the work left after the routing: the routed
    // tasks, and on the down owners (CTAs [G - n_dt, G)) their down records,
    // which stream in the same rings meanwhile.  The logits and the shared
    // gate/up tasks ran before the routing and do not count.  A CTA's share
    // of the tasks is its capacity's share of the total, rounded the same way
    // in every CTA (monotone in the CTA index).
    if (lane == 0) {
      const int nr_total = U * pl.rbg;
      const int64_t task_w = pl.nch_d * 10;
      const int64_t down_w = int64_t(U * pl.nch_i + lay.nch_s) * 5;
      const int b2 = G - pl.n_dt;
      const int64_t target = (int64_t(pl.n_dt) * down_w + int64_t(nr_total) * task_w) / G;
      const int64_t cap_own = target > down_w ? target - down_w : 0;
      auto cum_cap = [&](int c) -> int64_t {
        return int64_t(min(c, b2)) * target + int64_t(max(0, c - b2)) * cap_own;
      };
      const int64_t cap_tot = cum_cap(G), c_lo = cum_cap(int(blockIdx.x)), c_hi = cum_cap(int(blockIdx.x) + 1);
      int first, last;
      if (cap_tot > 0) {
        first = int((c_lo * nr_total + cap_tot / 2) / cap_tot);
        last = int((c_hi * nr_total + cap_tot / 2) / cap_tot);
        if (int(blockIdx.x) == G - 1) last = nr_total;
      } else {
        first = int(blockIdx.x) * nr_total / G;
        last = (int(blockIdx.x) + 1) * nr_total / G;
      }
      tb.plan[kPlanFirst] = first;
      tb.plan[kPlanNr] = last - first;
    }
  }
  __syncthreads();
  pl.U = tb.plan[kPlanU];
  pl.first = tb.plan[kPlanFirst];
  pl.nr = tb.plan[kPlanNr];
  pl.routed = true;
  if (blockIdx.x == 0) {
    if (a.inds_out)
      for (int i = threadIdx.x; i < pl.P; i += kDecThreads) a.inds_out[i] = tb.inds[i];
    if (a.w_out)
      for (int i = threadIdx.x; i < pl.P; i += kDecThreads) a.w_out[i] = tb.wts[i];
  }

  // ---- phase G: routed gate/up tasks
  ring_fill(a, pl, tb, rg, warp, pol);
  run_gu(1, pl.nr);

  // ---- barrier 2: every h row stored (run_gu ends with a CTA barrier)
  ring_fill(a, pl, tb, rg, warp, pol);
  if (threadIdx.x == 0) grid_arrive(a.sync + 1);

  if (pl.td < 0) {
    if (rg.timed_out) atomicOr(a.err, 0x100);
    return;   // no down tile (and nothing in flight): done
  }
  if (threadIdx.x == 0) {
    if (!grid_wait(a.sync + 1, uint32_t(G), a.wait_ns)) {
      atomicOr(a.err, 0x400);
      tb.plan[kPlanAbort] = 1;
    }
  }
  __syncthreads();
  if (tb.plan[kPlanAbort]) {
    ring_drain(rg);
    if (sd_owner && threadIdx.x == 0) mbar_wait(sd_bar, 0);
    return;
  }

  // ---- h records of every position
  {
    const int n = lay.Pp * lay.nch_h * 16;
    for (int i = threadIdx.x; i < ((n + 31) & ~31); i += kDecThreads) {
      const bool live0 = i < n;
      const int pos = live0 ? i / (lay.nch_h * 16) : 0;
      const int r = live0 ? i - pos * lay.nch_h * 16 : 0;
      const int ch = r >> 4, blk = r & 15;
      const int K = pos >= pl.P ? a.Is : a.I;
      const bool live = live0 && ch * 128 < K;
      const uint4 v = live ? __ldcg(reinterpret_cast<const uint4*>(a.h + int64_t(pos) * a.ldh + ch * 128 + blk * 8))
                           : make_uint4(0, 0, 0, 0);
      put_record_block(smem + lay.off_h + (ch * lay.Pp + pos) * kActRecord, blk, v, live);
    }
  }
  __syncthreads();

  // ---- phase D: this CTA's 16 rows of the down projection, one expert a
  // job: jobs u = warp, warp + 8, ... (the shared expert last)
  {
    uint16_t* ydn = reinterpret_cast<uint16_t*>(smem + lay.off_y);
    const int ndj = pl.U + (a.Is > 0 ? 1 : 0);
    for (int u = warp; u < ndj; u += kDecWarps) {
      const bool sh = u == pl.U;
      const int p0 = sh ? pl.P : tb.p0[u];
      const int cnt = sh ? T : tb.cnt[u];
      const int nch = sh ? lay.nch_s : pl.nch_i;
      uint32_t tokoff[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) tokoff[q] = uint32_t(p0 + q) * kActRecord;
      float acc[1][2][2] = {};
      if (sh && !mbar_wait(sd_bar, 0)) rg.timed_out = true;
      for (int ch = 0; ch < nch; ++ch) {
        uint32_t st;
        if (sh) {
          st = smem_u32(smem + lay.off_sd) + ch * 1280;
        } else {
          if (rg.issued - rg.used < rg.R && rg.cur.ph != 3) ring_fill(a, pl, tb, rg, warp, pol);
          st = ring_take(rg);
        }
        const uint32_t brec = smem_u32(smem + lay.off_h) + ch * lay.Pp * kActRecord;
        if (cnt > 2)
          rec_mma<2, 1>(st, brec, tokoff, cnt, zaddr, acc);
        else
          rec_mma<1, 1>(st, brec, tokoff, cnt, zaddr, acc);
        if (!sh) ring_release(rg);
      }
#pragma unroll
      for (int q = 0; q < 2; ++q)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const float v = acc[0][q][h] + __shfl_xor_sync(0xFFFFFFFFu, acc[0][q][h], 1);
          const int j = 2 * q + ((lane & 3) >> 1);
          if ((lane & 1) == 0 && j < cnt) ydn[(p0 + j) * lay.tile_rows + (lane >> 2) + 8 * h] = f32_to_bf16(v);
        }
    }
  }
  __syncthreads();

  // ---- combine of this CTA's rows (combine_kernel's order)
  {
    const uint16_t* ydn = reinterpret_cast<const uint16_t*>(smem + lay.off_y);
    for (int i = threadIdx.x; i < T * lay.tile_rows; i += kDecThreads) {
      const int t = i / lay.tile_rows, r = i - t * lay.tile_rows;
      const int row = pl.td * lay.tile_rows + r;
      if (row >= d) continue;
      float acc = 0.f;
      for (int s = 0; s < k; ++s) {
        const int pos = tb.posof[t * k + s];
        if (pos < 0) continue;   // a dropped id
        const float w = bf16_to_f32(tb.wts[t * k + s]);
        acc = __fadd_rn(acc, __fmul_rn(bf16_to_f32(ydn[pos * lay.tile_rows + r]), w));
      }
      float out = bf16r(acc);
      if (a.Is > 0) {
        const float gate = bf16_to_f32(__ldcg(a.sg + t));
        const float s0 = bf16r(__fmul_rn(bf16_to_f32(ydn[(pl.P + t) * lay.tile_rows + r]), gate));
        out = bf16r(__fadd_rn(out, s0));
      }
      a.y[int64_t(t) * d + row] = f32_to_bf16(out);
    }
  }
  if (rg.timed_out) atomicOr(a.err, 0x100);
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------

static int dec_smem_cap() {
  static int cap[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  if (cap[dev] == 0) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess) v = 0;
    // room for the static shared memory
    cap[dev] = v > 4096 ? v - 1024 : 0;
  }
  return cap[dev];
}

bool decode_supported(int T, int E, int d, int k, int I, int Is, int gu_tile_rows, int dn_tile_rows) {
  if (T < 1 || T > kDecodeMaxT || T * k > kDecMaxRoutes || k > kMaxK) return false;
  if (E < 1 || E > 1024 || d % 128 || I % 128 || (Is && Is % 128) || d > 8192) return false;
  if (gu_tile_rows != 16 || (dn_tile_rows != 16 && dn_tile_rows != 32)) return false;
  const int G = sm_count();
  const int L = (E + kDecLogitRows - 1) / kDecLogitRows;
  const int n_dt = (d + 15) / 16;            // 16-row owners of y
  if (L >= G || n_dt > G) return false;   // CTA L computes the shared gate
  const int cap = dec_smem_cap();
  if (cap <= 0) return false;
  const DecLayout lay = dec_layout(T, d, k, I, Is, dn_tile_rows / 16, cap);
  // enough stages to keep every warp's stream going
  return lay.ring_stages >= 2 * kDecWarps && lay.total <= cap;
}

template <int PER, int DNMT>
static cudaError_t launch_decode_t(const DecodeArgs& a0, cudaStream_t st) {
  DecodeArgs a = a0;
  a.smem_bytes = dec_smem_cap();
  const DecLayout lay = dec_layout(a.T, a.d, a.k, a.I, a.Is, DNMT, a.smem_bytes);
  auto kern = decode_kernel<PER, DNMT>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, lay.total);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(sm_count());
  cfg.blockDim = dim3(kDecThreads);
  cfg.dynamicSmemBytes = lay.total;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, a);
}

template <int PER>
static cudaError_t launch_decode_p(const DecodeArgs& a, cudaStream_t st) {
  return a.dn_mt == 2 ? launch_decode_t<PER, 2>(a, st) : launch_decode_t<PER, 1>(a, st);
}

cudaError_t launch_decode(const DecodeArgs& a, cudaStream_t st) {
  if (a.dn_mt != 1 && a.dn_mt != 2) return cudaErrorInvalidValue;
  const int per = (a.E + 31) / 32;
  if (per <= 4) return launch_decode_p<4>(a, st);
  if (per <= 8) return launch_decode_p<8>(a, st);
  if (per <= 16) return launch_decode_p<16>(a, st);
  return launch_decode_p<32>(a, st);
}

}  // namespace vx
