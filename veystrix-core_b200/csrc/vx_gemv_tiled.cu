// Grouped Q4 GEMV over the tiled expert pool (sm_100a).
//
// The MLX-layout kernel's scheme (vx_gemv_mma.cu: mma.sync m16n8k16 with the
// block-diagonal B, MLX's qmv formula per group folded into the epilogue),
// but every operand arrives by copies from records laid out in the order
// the warp consumes them.  Both passes read act_records_kernel's f16 records
// (x for gate/up, h for down) and unpack the nibbles to f16 subnormals
// q * 2^-24 and 16q * 2^-24 by one mask per pair and one shift per word (the
// kernel is bound by the ALU pipe, and the unpack is most of its ALU work);
// the products q * x are exact.  (The bf16 128 + q unpack by one lop3 and a
// shift per pair, with the group sums formed on the tensor pipe, remains for
// bf16 records without sums: kActF16 false.)
//
// Weight records (the pool, re-tiled once at load time).  One record = one
// warp's 128-input chunk of one row tile:
//
//   [p][m][h][lane] 16 B   packed words: lane (g = lane/4, c = lane%4) gets
//                          row 16m + g + 8h of the tile, words 4c..4c+3
//   [p][m][g][c&1] 16 B    {scale, bias} of groups 4ch+2(c&1) and +1 for rows
//                          g and g+8, as bf16 pairs {s_a s_b | b_a b_b} per row
//
// (p: projection - gate and up interleaved for the gate/up pass; m: 16-row
// m-tile).  1280 bytes per (p, m): 1024 of weights, 256 of scales and biases,
// the same bytes as the MLX layout.  Expert e's records start at e * stride,
// the counterpart of the reference's fixed-stride expert records
// (models/flashnext/slab_pack.py:1-25, expert_pool.py:1-22).
//
// Activation records (written per call): per (chunk, sorted position) the
// chunk's 128 inputs in lane order plus the group sums (kActRecord bytes).
// An item's positions are consecutive, so lane 0 brings a chunk's weights
// and all of the item's activations with two bulk copies onto one mbarrier;
// no other lane issues copies or computes addresses.
//
// Items hold up to four tokens: B operand 0 carries tokens 0-1, B operand 1
// tokens 2-3 (only for items with more than two), both multiplied against
// the same unpacked weight fragments.  The pipeline runs across the warp's
// tasks, so the copies of the next task start while the current one is
// being consumed.  Records out of range (rows >= out, groups >= in/32) hold
// zeros and add exactly zero.
#include <cuda_fp16.h>

#include <type_traits>

#include "vx_async.cuh"
#include "vx_common.cuh"
#include "vx_launch.h"

namespace vx {

constexpr int kTiledWarps = 8;
constexpr int kTiledStages = 3;
// Decode-sized batches have too few (item, row tile) tasks to fill the GPU
// with warps: each warp then walks its task's chunks with a deep pipeline
// (kDeepStages - 1 chunks in flight instead of kTiledStages - 1) in 4-warp
// CTAs, one task per warp.
constexpr int kDeepStages = 8;
constexpr int kDeepWarps = 4;
// Resident CTAs per SM of a GEMV shape: the deep one alone, the others two.
__host__ __device__ constexpr int tiled_ctas_per_sm(int stages, int warps) {
  return (stages == kDeepStages && warps == kDeepWarps) ? 1 : 2;
}

struct TiledTask {
  int e, p0, cnt, row0, N, K;
  bool sh;
};

template <int MT>
VX_DEVICE bool decode_task(const TiledArgs& a, int t, TiledTask& k) {
  const int item = t / a.tiles_per_item, rb = t - item * a.tiles_per_item;
  k.e = __ldg(a.items + 3 * item);
  k.p0 = __ldg(a.items + 3 * item + 1);
  k.cnt = __ldg(a.items + 3 * item + 2);
  k.sh = k.e == a.E;
  k.N = k.sh ? a.N_s : a.N_b;
  k.K = k.sh ? a.K_s : a.K_b;
  k.row0 = rb * 16 * MT;
  return k.row0 < k.N;
}

// Lane 0 arms the stage's mbarrier for both copies and issues them; the
// other lanes execute nothing (predicated inside one asm block, no branch).
VX_DEVICE void issue_stage(bool leader, uint32_t bar, uint32_t dst_w, const void* src_w, uint32_t nw,
                           uint64_t pol_w, uint32_t dst_x, const void* src_x, uint32_t nx,
                           uint64_t pol_x) {
  asm volatile(
      "{\n"
      ".reg .pred p;\n"
      "setp.ne.b32 p, %0, 0;\n"
      "@p fence.proxy.async.shared::cta;\n"
      "@p mbarrier.arrive.expect_tx.shared::cta.b64 _, [%1], %2;\n"
      "@p cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%3], [%4], %5, "
      "[%1], %6;\n"
      "@p cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%7], [%8], %9, "
      "[%1], %10;\n"
      "}\n" ::"r"(int(leader)),
      "r"(bar), "r"(nw + nx), "r"(dst_w), "l"(src_w), "r"(nw), "l"(pol_w), "r"(dst_x), "l"(src_x), "r"(nx),
      "l"(pol_x)
      : "memory");
}

// Lane 0 arms the stage's mbarrier for the activation copy alone and issues
// it (the weights travel by per-lane cp.async, see below).
VX_DEVICE void issue_act(bool leader, uint32_t bar, uint32_t dst_x, const void* src_x, uint32_t nx,
                         uint64_t pol_x) {
  asm volatile(
      "{\n"
      ".reg .pred p;\n"
      "setp.ne.b32 p, %0, 0;\n"
      "@p fence.proxy.async.shared::cta;\n"
      "@p mbarrier.arrive.expect_tx.shared::cta.b64 _, [%1], %2;\n"
      "@p cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%3], [%4], %2, "
      "[%1], %5;\n"
      "}\n" ::"r"(int(leader)),
      "r"(bar), "r"(nx), "r"(dst_x), "l"(src_x), "l"(pol_x)
      : "memory");
}

// The weight records travel through the load/store units (each lane copies
// 16-byte pieces with cp.async) while the small activation records use the
// bulk-copy engine: one SM's bulk-copy (TMA) engine alone sustains about 14
// bytes per cycle - about 4 TB/s over the chip - below what HBM delivers,
// so the heavy stream goes the other way.
constexpr bool kWeightsByLsu = true;

// Depth of the per-warp task queue from producer to consumer: the producer
// runs at most STAGES - 1 records (so as many tasks) ahead.
constexpr int kTaskFifo = 16;

template <bool GATEUP, int MT, bool XMMA, int STAGES, int WARPS, int GS>
__global__ void __launch_bounds__(WARPS * 32, tiled_ctas_per_sm(STAGES, WARPS))
    gemv_tiled_kernel(const __grid_constant__ TiledArgs a) {
  chain_wait();
  constexpr int NP = GATEUP ? 2 : 1;
  // gate/up reads act_records_kernel's f16 records; down reads h in bf16
  constexpr bool F16 = kActF16;
  constexpr int kRec = NP * MT * tile_unit_bytes(GS);
  constexpr int kSbUnit = tile_unit_bytes(GS) - 1024;   // scale/bias bytes per (p, m)
  constexpr int kWBytes = NP * MT * 1024;
  constexpr int kXOff = kRec;                       // [token][kActRecord]
  constexpr int kStage = kRec + kTiledItemChunk * kActRecord;
  static_assert(kStage % 128 == 0, "stage size");
  static_assert(STAGES < kTaskFifo, "task queue depth");
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ __align__(8) uint64_t bars[WARPS][STAGES];
  __shared__ __align__(16) uint32_t zero16[4];
  // tasks from the producer cursor to the consumer, in issue order (-1: end)
  __shared__ int tfifo[WARPS][kTaskFifo];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;
  if (threadIdx.x < 4) zero16[threadIdx.x] = 0u;
  if (lane == 0)
    for (int s = 0; s < STAGES; ++s) mbar_init(smem_u32(&bars[warp][s]));
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  __syncthreads();
  const uint32_t ring = smem_u32(smem) + warp * STAGES * kStage;
  const uint32_t bar0 = smem_u32(&bars[warp][0]);
  const uint32_t zaddr = smem_u32(zero16);
  const bool blane = (g & 3) == c;   // carries token (g >> 2) of its pair on group c
  const int tb = g >> 2, ts = c >> 1;
  const int n_items = *a.n_items;
  const int total = n_items * a.tiles_per_item;
  const int nw = gridDim.x * WARPS;
  const uint64_t pol_w = policy_evict_first();
  const uint64_t pol_x = policy_evict_last();
  const int64_t act_pitch = a.act_rows * kActRecord;   // bytes per chunk of activations

  // ---- producer cursor: task ti, chunk ci ----
  // The first wave is static (task = global warp index); later tasks come
  // from a.task_ctr in the order warps ask, so a warp whose tasks ran short
  // (one-token items) takes more of them.  Lane 0 asks one task ahead: the
  // atomic's latency hides behind a whole task.
  int ti = blockIdx.x * WARPS + warp, ci = 0;
  const bool dyn = a.task_ctr != nullptr;
  int tnext = 0;
  if (dyn && lane == 0) tnext = atomicAdd(a.task_ctr, 1);
  auto advance = [&]() {
    if (dyn) {
      ti = nw + __shfl_sync(0xFFFFFFFFu, tnext, 0);
      if (lane == 0) tnext = atomicAdd(a.task_ctr, 1);
    } else {
      ti += nw;
    }
  };
  int qt = 0;   // tasks pushed to tfifo
  int inch = 0;
  uint32_t ixbytes = 0;
  const unsigned char* irec = nullptr;
  const unsigned char* iact = nullptr;
  auto seek = [&]() {   // first valid task at or after ti
    for (; ti < total; advance()) {
      TiledTask k;
      if (!decode_task<MT>(a, ti, k)) continue;
      const int rb = k.row0 / (16 * MT);
      inch = (k.K + 127) >> 7;
      irec = (k.sh ? a.rec_s : a.rec_b + routed_record(a.slot_of, a.slots, k.e) * a.stride_b) +
             int64_t(rb) * inch * kRec;
      iact = a.act + int64_t(k.p0) * kActRecord;
      ixbytes = uint32_t(k.cnt) * kActRecord;
      tfifo[warp][qt++ % kTaskFifo] = ti;   // every lane writes the same value
      return;
    }
    tfifo[warp][qt++ % kTaskFifo] = -1;
  };
  int st_issue = 0, st_use = 0;
  uint32_t parity_bits = 0;   // bit s: parity expected next on stage s
  bool timed_out = false;
  auto issue = [&]() {
    const uint32_t st = ring + st_issue * kStage;
    if (kWeightsByLsu) {
      const unsigned char* src = irec + int64_t(ci) * kRec + lane * 16;
#pragma unroll
      for (int j = 0; j < (kRec + 511) / 512; ++j)
        cp16_if(st + j * 512 + lane * 16, src + j * 512, 16, j * 512 + lane * 16 < kRec);
      issue_act(lane == 0, bar0 + 8 * st_issue, st + kXOff, iact + int64_t(ci) * act_pitch, ixbytes, pol_x);
    } else {
      issue_stage(lane == 0, bar0 + 8 * st_issue, st, irec + int64_t(ci) * kRec, kRec, pol_w, st + kXOff,
                  iact + int64_t(ci) * act_pitch, ixbytes, pol_x);
    }
    st_issue = st_issue == STAGES - 1 ? 0 : st_issue + 1;
    if (++ci == inch) {
      ci = 0;
      advance();
      seek();
    }
  };

  seek();
#pragma unroll
  for (int s = 0; s < STAGES - 1; ++s) {
    if (ti < total) issue();
    cp_commit();   // one cp.async group per unit, empty ones included
  }

  // ---- consumer: tasks in the same order ----
  auto run = [&](const TiledTask& k, auto nq_tag) {
    constexpr int NQ = decltype(nq_tag)::value;   // B operands (token pairs)
    float acc[NP][MT][NQ][2];
#pragma unroll
    for (int p = 0; p < NP; ++p)
#pragma unroll
      for (int m = 0; m < MT; ++m)
#pragma unroll
        for (int q = 0; q < NQ; ++q) acc[p][m][q][0] = acc[p][m][q][1] = 0.f;
    // B lanes of a present token read its activations; the others read zeros
    uint32_t xa[NQ], xsa[NQ];
#pragma unroll
    for (int q = 0; q < NQ; ++q) {
      const bool live = blane && 2 * q + tb < k.cnt;
      xa[q] = live ? kXOff + (2 * q + tb) * kActRecord + c * 16 : 0xFFFFFFFFu;
      xsa[q] = kXOff + (2 * q + ts) * kActRecord + kActXsum + (c & 1) * 8;
    }
    // 2^(24-e) of the lane's token (f16 records: the chunks accumulate on the
    // records' scaled axis, scaled back once after the last chunk)
    float xinv[NQ] = {};
    const int nch = (k.K + 127) >> 7;
    for (int ch = 0; ch < nch; ++ch) {
      if (ti < total) issue();
      cp_commit();
      const uint32_t st = ring + st_use * kStage;
      if (kWeightsByLsu) {
        cp_wait<STAGES - 1>();   // this unit's weight pieces (every lane's)
        __syncwarp();
      }
      if (!mbar_wait(bar0 + 8 * st_use, (parity_bits >> st_use) & 1u)) timed_out = true;
      parity_bits ^= 1u << st_use;

      uint32_t bq[NQ][16];
      float xs[NQ][2];
#pragma unroll
      for (int q = 0; q < NQ; ++q) {
        const bool live = xa[q] != 0xFFFFFFFFu;
        const uint32_t base = live ? st + xa[q] : zaddr;
        const uint32_t step = live ? 64 : 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const uint4 v = lds128(base + i * step);
          bq[q][4 * i + 0] = v.x;
          bq[q][4 * i + 1] = v.y;
          bq[q][4 * i + 2] = v.z;
          bq[q][4 * i + 3] = v.w;
        }
        if (XMMA) {
          float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int mm = 0; mm < 8; ++mm)
            mma16816(d, 0x3F803F80u, 0x3F803F80u, 0x3F803F80u, 0x3F803F80u, bq[q][2 * mm], bq[q][2 * mm + 1]);
          xs[q][0] = d[0];
          xs[q][1] = d[1];
        } else if (F16) {
          const uint2 v = lds64(st + xsa[q]);
          xs[q][0] = __uint_as_float(v.x);
          xs[q][1] = __uint_as_float(v.y);
          xinv[q] = __uint_as_float(lds64(st + xsa[q] - (c & 1) * 8 + 16).x);
        } else {
          const uint2 v = lds64(st + xsa[q]);
          xs[q][0] = __uint_as_float(v.x);
          xs[q][1] = __uint_as_float(v.y);
        }
      }
#pragma unroll
      for (int p = 0; p < NP; ++p) {
#pragma unroll
        for (int m = 0; m < MT; ++m) {
          const uint32_t wrow = st + (p * MT + m) * 1024 + lane * 16;
          const uint4 wg = lds128(wrow), w8 = lds128(wrow + 512);
          const uint32_t ag[4] = {wg.x, wg.y, wg.z, wg.w};
          const uint32_t a8[4] = {w8.x, w8.y, w8.z, w8.w};
          float d[NQ][4];
#pragma unroll
          for (int q = 0; q < NQ; ++q)
#pragma unroll
            for (int i = 0; i < 4; ++i) d[q][i] = 0.f;
#pragma unroll
          for (int mm = 0; mm < 8; mm += 2) {
            const int wi = mm >> 1;
            if constexpr (F16) {
              // four masks and one shift per word: f16 subnormals q * 2^-24
              // (f0 f1 h0 h1) and 16q * 2^-24 (f2 f3 h2 h3, against B rows
              // k >= 8, whose activations are stored / 16)
              const uint32_t g8 = ag[wi] >> 8, e8 = a8[wi] >> 8;
              const uint32_t f0 = ag[wi] & 0x000F000Fu, f1 = a8[wi] & 0x000F000Fu;
              const uint32_t f2 = ag[wi] & 0x00F000F0u, f3 = a8[wi] & 0x00F000F0u;
              const uint32_t h0 = g8 & 0x000F000Fu, h1 = e8 & 0x000F000Fu;
              const uint32_t h2 = g8 & 0x00F000F0u, h3 = e8 & 0x00F000F0u;
#pragma unroll
              for (int q = 0; q < NQ; ++q) {
                mma16816_f16(d[q], f0, f1, f2, f3, bq[q][2 * mm], bq[q][2 * mm + 1]);
                mma16816_f16(d[q], h0, h1, h2, h3, bq[q][2 * mm + 2], bq[q][2 * mm + 3]);
              }
              continue;
            }
            const uint32_t f0 = nib_pair128(ag[wi]), f1 = nib_pair128(a8[wi]);
            const uint32_t f2 = nib_pair128(ag[wi] >> 4), f3 = nib_pair128(a8[wi] >> 4);
            const uint32_t h0 = nib_pair128(ag[wi] >> 8), h1 = nib_pair128(a8[wi] >> 8);
            const uint32_t h2 = nib_pair128(ag[wi] >> 12), h3 = nib_pair128(a8[wi] >> 12);
#pragma unroll
            for (int q = 0; q < NQ; ++q) {
              // one accumulator chain per B operand, in the MLX-layout kernel's order
              mma16816(d[q], f0, f1, f2, f3, bq[q][2 * mm], bq[q][2 * mm + 1]);
              mma16816(d[q], h0, h1, h2, h3, bq[q][2 * mm + 2], bq[q][2 * mm + 3]);
            }
          }
          uint32_t sw[4];
          if constexpr (GS == 64) {
            // one {s | b} per row: groups 2(c&1) and 2(c&1)+1 share it
            const uint2 sb = lds64(st + kWBytes + (p * MT + m) * kSbUnit + (g * 2 + (c & 1)) * 8);
            sw[0] = (sb.x & 0xFFFFu) * 0x10001u;
            sw[1] = (sb.x >> 16) * 0x10001u;
            sw[2] = (sb.y & 0xFFFFu) * 0x10001u;
            sw[3] = (sb.y >> 16) * 0x10001u;
          } else {
            const uint4 sb = lds128(st + kWBytes + (p * MT + m) * kSbUnit + (g * 2 + (c & 1)) * 16);
            sw[0] = sb.x;
            sw[1] = sb.y;
            sw[2] = sb.z;
            sw[3] = sb.w;
          }
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const float s0 = __uint_as_float(sw[2 * h] << 16);
            const float s1 = __uint_as_float(sw[2 * h] & 0xFFFF0000u);
            const float b0 = __uint_as_float(sw[2 * h + 1] << 16);
            const float b1 = __uint_as_float(sw[2 * h + 1] & 0xFFFF0000u);
            if constexpr (F16) {
#pragma unroll
              for (int q = 0; q < NQ; ++q) {
                float v = acc[p][m][q][h];
                v = fmaf(s0, d[q][2 * h], v);
                v = fmaf(b0, xs[q][0], v);
                v = fmaf(s1, d[q][2 * h + 1], v);
                v = fmaf(b1, xs[q][1], v);
                acc[p][m][q][h] = v;
              }
              continue;
            }
            // bias - 128*scale: the lop3 operands carry q + 128.
            const float c0 = fmaf(-128.f, s0, b0);
            const float c1 = fmaf(-128.f, s1, b1);
#pragma unroll
            for (int q = 0; q < NQ; ++q) {
              float v = acc[p][m][q][h];
              v = fmaf(s0, d[q][2 * h], v);
              v = fmaf(c0, xs[q][0], v);
              v = fmaf(s1, d[q][2 * h + 1], v);
              v = fmaf(c1, xs[q][1], v);
              acc[p][m][q][h] = v;
            }
          }
        }
      }
      __syncwarp();   // the stage is read out before the warp refills it
      st_use = st_use == STAGES - 1 ? 0 : st_use + 1;
    }

    // lanes c and c^1 hold the two group halves of the same (row, token)
#pragma unroll
    for (int p = 0; p < NP; ++p)
#pragma unroll
      for (int m = 0; m < MT; ++m)
#pragma unroll
        for (int q = 0; q < NQ; ++q)
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            acc[p][m][q][h] += __shfl_xor_sync(0xFFFFFFFFu, acc[p][m][q][h], 1);
            if constexpr (F16) acc[p][m][q][h] *= xinv[q];   // lanes c, c^1: the same token
          }
    if (c & 1) return;
#pragma unroll
    for (int q = 0; q < NQ; ++q) {
      const int tok = 2 * q + (c >> 1);
      if (tok >= k.cnt) continue;
      const int64_t pos = k.p0 + tok;
#pragma unroll
      for (int m = 0; m < MT; ++m)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int row = k.row0 + 16 * m + g + 8 * h;
          if (row >= k.N) continue;
          if (GATEUP) {
            // h, the down projection's input, as plain rows (its f16 records
            // need the largest |h| of each 128 rows, from other tasks)
            const float v = silu_mul_bf16(bf16r(acc[0][m][q][h]), bf16r(acc[NP - 1][m][q][h]));
            a.out[pos * a.ldo + row] = f32_to_bf16(v);
          } else {
            a.out[pos * a.ldo + row] = f32_to_bf16(acc[0][m][q][h]);
          }
        }
    }
  };

  for (int qh = 0;; ++qh) {
    const int t = tfifo[warp][qh % kTaskFifo];   // written by this lane in seek()
    if (t < 0) break;
    TiledTask k;
    decode_task<MT>(a, t, k);   // a valid task (seek() skips the others)
    if (kTiledItemChunk > 2 && k.cnt > 2)
      run(k, std::integral_constant<int, 2>());
    else
      run(k, std::integral_constant<int, 1>());
  }
  cp_wait<0>();
  if (timed_out && a.err) atomicOr(a.err, 0x100);
}

// ---- activation records ----------------------------------------------------

// One CTA per position; thread i writes 8-input blocks i, i + blockDim, ...
// of the position's records (a record's 16 blocks are 16 consecutive lanes).  The
// block goes to lane-order slot (i*4 + c) in B order (words (x0,x4) (x1,x5)
// (x2,x6) (x3,x7)) as f16, for the f16 unpack of the GEMV (kActF16; x rows
// for gate/up, h rows for down), whose weights enter the MMA as f16
// subnormals q * 2^-24 (nibbles at bits 0-3) or 16q * 2^-24 (bits 4-7, no
// shift):
//
//   * all records of a position are scaled by 2^e, e chosen from the
//     position's largest |x| so that it lands in [2^13, 2^14): every bf16
//     input converts exactly (f16 keeps 11 significant bits) unless it is
//     2^-27 of the largest or smaller (then to the nearest multiple of
//     2^-24 on the scaled axis, an error below 2^-38 of the largest);
//   * words 1 and 3 of each slot meet the 16q weights (B rows k = 8..15 of
//     an MMA): those values are stored divided by 16 (exact), so every
//     product is q * x * 2^(e-24);
//   * the tail holds the sum of each group's 32 inputs times 2^(e-24) at
//     kActXsum + 4g (left to right over 8 inputs, then (s0+s1)+(s2+s3), then
//     the exact scaling), for the bias term, and 2^(24-e) at kActXsum + 16.
//
// A group's GEMV term on the scaled axis is s * D + b * sum', D the MMA sum:
// exact products and an fp32 sum with no offset to cancel; the task's sum
// over its chunks is multiplied by 2^(24-e) once, which gives the same bits
// as scaling every term (a power of two commutes with rounding while the
// values stay normal).  e stays at or above -103 so that 2^(24-e) is a
// finite float: a position whose largest |x| is 2^117 or more saturates to
// infinity.
// E with m in [2^(E-1), 2^E), for a positive finite float (subnormals too):
// from the exponent field, or for a subnormal the position of its leading bit.
VX_DEVICE int pow2_exponent(float m) {
  const uint32_t b = __float_as_uint(m);
  const int ex = int(b >> 23);
  return ex ? ex - 126 : (31 - __clz(int(b))) - 148;
}

// x * 2^n for n in [-190, 254], by multiplying with exact powers of two (one
// rounding, as a scaling by 2^n is exact whenever the result is normal).
VX_DEVICE float times_pow2(float x, int n) {
  if (n > 127) {
    x *= __int_as_float((64 + 127) << 23);
    n -= 64;
  } else if (n < -126) {
    x *= __int_as_float((127 - 64) << 23);
    n += 64;
  }
  return x * __int_as_float((n + 127) << 23);
}

constexpr int kActThreads = 256;

__global__ void act_records_kernel(const uint16_t* __restrict__ x, int64_t ldx, int K,
                                   const int32_t* __restrict__ src_rows, const int32_t* __restrict__ n_rows,
                                   int64_t rows, unsigned char* __restrict__ act) {
  chain_begin();
  // one CTA per position: the exponent comes from the whole row's largest
  // |x|, so every chunk of a position shares it (the GEMV accumulates the
  // chunks on the scaled axis and scales once per task)
  __shared__ float wmax[kActThreads / 32];
  const int nb = ((K + 127) / 128) * 16;   // 8-input blocks, chunk padding included
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t p = blockIdx.x;
  if (p >= (n_rows ? int64_t(*n_rows) : rows)) return;   // CTA-uniform
  const uint16_t* xr = x + (src_rows ? int64_t(__ldg(src_rows + p)) : p) * ldx;
  float m = 0.f;
  uint4 v0 = make_uint4(0, 0, 0, 0);   // the first round's block, kept for the second pass
  for (int blk = threadIdx.x; blk * 8 < K; blk += blockDim.x) {
    const uint4 v = *reinterpret_cast<const uint4*>(xr + blk * 8);
    if (blk == int(threadIdx.x)) v0 = v;
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int j = 0; j < 4; ++j)
      m = fmaxf(m, fmaxf(fabsf(__uint_as_float(w[j] << 16)), fabsf(__uint_as_float(w[j] & 0xFFFF0000u))));
  }
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) m = fmaxf(m, __shfl_xor_sync(0xFFFFFFFFu, m, o));
  if (lane == 0) wmax[warp] = m;
  __syncthreads();
  m = wmax[0];
  for (int i = 1; i < int(blockDim.x >> 5); ++i) m = fmaxf(m, wmax[i]);
  int e = 0;
  if (m > 0.f && isfinite(m)) e = max(14 - pow2_exponent(m), -103);
  for (int b0 = 0; b0 < nb; b0 += blockDim.x) {   // uniform over the CTA
    const int blk = b0 + threadIdx.x;
    const bool inside = blk * 8 < K;   // implies blk < nb
    uint4 v = b0 == 0 ? v0 : make_uint4(0, 0, 0, 0);
    if (inside && b0 > 0) v = *reinterpret_cast<const uint4*>(xr + blk * 8);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    float xv[8];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      xv[2 * j] = __uint_as_float(w[j] << 16);
      xv[2 * j + 1] = __uint_as_float(w[j] & 0xFFFF0000u);
    }
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) s += xv[j];
    s += __shfl_xor_sync(0xFFFFFFFFu, s, 1);
    s += __shfl_xor_sync(0xFFFFFFFFu, s, 2);
    if (blk >= nb) continue;
    const int ch = blk >> 4, c = (blk >> 2) & 3, ib = blk & 3;
    unsigned char* rec = act + (int64_t(ch) * rows + p) * kActRecord;
    uint16_t h[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) h[j] = __half_as_ushort(__float2half_rn(times_pow2(xv[j], (j & 1) ? e - 4 : e)));
    uint4 o;
    o.x = h[0] | (uint32_t(h[4]) << 16);   // (x0, x4)
    o.y = h[1] | (uint32_t(h[5]) << 16);   // (x1, x5) / 16: B rows k >= 8
    o.z = h[2] | (uint32_t(h[6]) << 16);   // (x2, x6)
    o.w = h[3] | (uint32_t(h[7]) << 16);   // (x3, x7) / 16
    *reinterpret_cast<uint4*>(rec + (ib * 4 + c) * 16) = o;
    // the group sum on the records' scale, 2^(e-24) (exact: a power of two)
    if (ib == 0) *reinterpret_cast<float*>(rec + kActXsum + c * 4) = times_pow2(s, e - 24);
    if ((blk & 15) == 0) *reinterpret_cast<float*>(rec + kActXsum + 16) = __int_as_float((24 - e + 127) << 23);
  }
}

cudaError_t launch_act_records(const uint16_t* x, int64_t ldx, int K, const int32_t* src_rows,
                               const int32_t* n_rows, int64_t rows, unsigned char* act,
                               cudaStream_t st) {
  if (rows <= 0 || K <= 0) return cudaSuccess;
  if (rows > 0x7FFFFFFF) return cudaErrorInvalidValue;
  const int nb = ((K + 127) / 128) * 16;   // threads: one per 8-input block, at most kActThreads
  const int threads = nb >= kActThreads ? kActThreads : (nb + 31) / 32 * 32;
  return launch_chained(act_records_kernel, dim3(unsigned(rows)), dim3(threads), 0, st, x, ldx, K,
                        src_rows, n_rows, rows, act);
}

// ---- pool packing -----------------------------------------------------------

// One thread per 16-byte unit of the pool.  a: first (or only) projection,
// b: second projection of a gate/up pair.  gs: the banks' quant group, 32
// ({s_a s_b | b_a b_b} per row pair and group pair) or 64 (native G64: one
// {s | b} word per row and 64 inputs, [g][c&1][h]).
__global__ void tile_pack_kernel(vx_q4 a, vx_q4 b, int NP, int MT, int RB, int nch, int gs, uint4* out,
                                 int64_t units) {
  const int per_rec = NP * MT * (tile_unit_bytes(gs) / 16);
  for (int64_t u = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; u < units;
       u += int64_t(gridDim.x) * blockDim.x) {
    const int64_t rec = u / per_rec;
    const int off = int(u - rec * per_rec);
    const int ch = int(rec % nch);
    const int rb = int((rec / nch) % RB);
    const int64_t e = rec / (int64_t(nch) * RB);
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (off < NP * MT * 64) {
      const int pm = off / 64, r = off % 64;
      const int h = r / 32, ln = r % 32;
      const int p = pm / MT, m = pm % MT;
      const vx_q4& bk = p ? b : a;
      const int row = rb * 16 * MT + 16 * m + (ln >> 2) + 8 * h;
      const int W = bk.in / 8;
      const int w0 = ch * 16 + 4 * (ln & 3);
      if (row < bk.out) {
        const uint32_t* src = bk.w + (e * bk.out + row) * W;
        v.x = w0 + 0 < W ? src[w0 + 0] : 0u;
        v.y = w0 + 1 < W ? src[w0 + 1] : 0u;
        v.z = w0 + 2 < W ? src[w0 + 2] : 0u;
        v.w = w0 + 3 < W ? src[w0 + 3] : 0u;
      }
    } else if (gs == 64) {
      // 8 units per (p, m): unit g holds {cb 0: row g, row g+8}{cb 1: ...}
      const int o2 = off - NP * MT * 64;
      const int pm = o2 / 8, g = o2 % 8;
      const int p = pm / MT, m = pm % MT;
      const vx_q4& bk = p ? b : a;
      const int G = bk.in / 64;
      uint32_t wd[4];
#pragma unroll
      for (int cb = 0; cb < 2; ++cb)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int row = rb * 16 * MT + 16 * m + g + 8 * h;
          const int gi = 2 * ch + cb;
          uint32_t sv = 0, bv = 0;
          if (row < bk.out && gi < G) {
            const int64_t idx = (e * bk.out + row) * G + gi;
            sv = bk.scales[idx];
            bv = bk.biases[idx];
          }
          wd[2 * cb + h] = sv | (bv << 16);
        }
      v = make_uint4(wd[0], wd[1], wd[2], wd[3]);
    } else {
      const int o2 = off - NP * MT * 64;
      const int pm = o2 / 16, q = o2 % 16;
      const int p = pm / MT, m = pm % MT;
      const vx_q4& bk = p ? b : a;
      const int gg = q >> 1, cb = q & 1;
      const int G = bk.in / bk.group_size;
      const int ga = 4 * ch + 2 * cb;
      uint32_t wd[4];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int row = rb * 16 * MT + 16 * m + gg + 8 * h;
        uint32_t sa = 0, sb = 0, ba = 0, bb = 0;
        if (row < bk.out) {
          const int64_t base = (e * bk.out + row) * G;
          if (ga < G) sa = bk.scales[base + ga], ba = bk.biases[base + ga];
          if (ga + 1 < G) sb = bk.scales[base + ga + 1], bb = bk.biases[base + ga + 1];
        }
        wd[2 * h] = sa | (sb << 16);
        wd[2 * h + 1] = ba | (bb << 16);
      }
      v = make_uint4(wd[0], wd[1], wd[2], wd[3]);
    }
    out[u] = v;
  }
}

int64_t tile_pool_bytes(int64_t experts, int out, int in, int nproj, int tile_rows, int group) {
  const int64_t RB = (out + tile_rows - 1) / tile_rows;
  const int64_t nch = (in + 127) / 128;
  return experts * RB * nch * int64_t(nproj) * (tile_rows / 16) * tile_unit_bytes(group);
}

cudaError_t launch_tile_pack(const vx_q4& a, const vx_q4& b, int nproj, int tile_rows, void* out,
                             cudaStream_t st, int group) {
  const int MT = tile_rows / 16;
  const int RB = (a.out + tile_rows - 1) / tile_rows;
  const int nch = (a.in + 127) / 128;
  const int64_t units = tile_pool_bytes(a.experts, a.out, a.in, nproj, tile_rows, group) / 16;
  if (units == 0) return cudaSuccess;
  int64_t blocks = (units + 255) / 256;
  if (blocks > int64_t(sm_count()) * 32) blocks = int64_t(sm_count()) * 32;
  tile_pack_kernel<<<int(blocks), 256, 0, st>>>(a, nproj == 2 ? b : a, nproj, MT, RB, nch, group,
                                                static_cast<uint4*>(out), units);
  return cudaGetLastError();
}

// ---- launcher ----------------------------------------------------------------

template <bool GATEUP, int MT, bool XMMA, int STAGES, int WARPS, int GS>
static cudaError_t launch_tiled_v(TiledArgs a, int64_t tasks, cudaStream_t st) {
  constexpr int NP = GATEUP ? 2 : 1;
  constexpr int kStage = NP * MT * tile_unit_bytes(GS) + kTiledItemChunk * kActRecord;
  const size_t smem = size_t(WARPS) * STAGES * kStage;
  auto kern = gemv_tiled_kernel<GATEUP, MT, XMMA, STAGES, WARPS, GS>;
  cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (err != cudaSuccess) return err;
  // persistent: two resident CTAs per SM for the 8-warp shape, one for the deep one
  const int64_t cap = int64_t(sm_count()) * tiled_ctas_per_sm(STAGES, WARPS);
  int64_t grid = (tasks + WARPS - 1) / WARPS;
  if (grid > cap) grid = cap;
  if (grid <= 0) return cudaSuccess;
  return launch_streaming(kern, dim3(int(grid)), dim3(WARPS * 32), smem, st, a);
}

template <bool GATEUP, int MT, bool XMMA, int GS>
static cudaError_t launch_tiled_t(TiledArgs a, int max_items, int max_out, cudaStream_t st) {
  a.tiles_per_item = (max_out + 16 * MT - 1) / (16 * MT);
  const int64_t tasks = int64_t(max_items) * a.tiles_per_item;
  // (a task with only a few chunks, as down's 4, gains nothing from the depth)
  if (tasks <= int64_t(sm_count()) * kDeepWarps && (a.K_b + 127) / 128 >= kDeepStages)
    return launch_tiled_v<GATEUP, MT, XMMA, kDeepStages, kDeepWarps, GS>(a, tasks, st);
  return launch_tiled_v<GATEUP, MT, XMMA, kTiledStages, kTiledWarps, GS>(a, tasks, st);
}

template <int GS>
static cudaError_t launch_gemv_tiled_g(bool gateup, int tile_rows, const TiledArgs& a, int max_items,
                                       int max_out, cudaStream_t st) {
  if (gateup) {
    if (tile_rows != 16) return cudaErrorInvalidValue;
    return launch_tiled_t<true, 1, false, GS>(a, max_items, max_out, st);
  }
  if (tile_rows == 32) return launch_tiled_t<false, 2, !kActF16, GS>(a, max_items, max_out, st);
  if (tile_rows == 16) return launch_tiled_t<false, 1, !kActF16, GS>(a, max_items, max_out, st);
  return cudaErrorInvalidValue;
}

// gate/up: activation records carry the group sums; the single projection
// (down) sums its input h on the tensor pipe.  group: the records' quant
// group (32, or 64 for native G64 records).
cudaError_t launch_gemv_tiled(bool gateup, int tile_rows, const TiledArgs& a, int max_items,
                              int max_out, cudaStream_t st, int group) {
  if (group == 64) return launch_gemv_tiled_g<64>(gateup, tile_rows, a, max_items, max_out, st);
  if (group == 32) return launch_gemv_tiled_g<32>(gateup, tile_rows, a, max_items, max_out, st);
  return cudaErrorInvalidValue;
}

}  // namespace vx
