// Grouped Q4 GEMV over the tiled expert pool (sm_100a).
//
// Same arithmetic as the MLX-layout kernel (vx_gemv_mma.cu: mma.sync
// m16n8k16 with the block-diagonal B, nibbles unpacked to 128+q by one lop3,
// MLX's qmv formula per group folded into the epilogue), but the weights come
// from a pool re-tiled once at load time into the order the warp consumes
// them.  One record = one warp's 128-input chunk of one row tile:
//
//   [p][m][h][lane] 16 B   packed words: lane (g = lane/4, c = lane%4) gets
//                          row 16m + g + 8h of the tile, words 4c..4c+3
//   [p][m][g][c&1] 16 B    {scale, bias} of groups 4ch+2(c&1) and +1 for rows
//                          g and g+8, as bf16 pairs {s_a s_b | b_a b_b} per row
//
// (p: projection - gate and up interleaved for the gate/up pass; m: 16-row
// m-tile).  1280 bytes per (p, m): 1024 of weights, 256 of scales and biases,
// the same bytes as the MLX layout.  A warp streams a row tile's records,
// which are contiguous, with ONE bulk copy per chunk (issued by lane 0,
// completed on the stage's mbarrier) instead of a TMA box plus eight small
// scale copies per lane.  The pipeline runs across the warp's tasks: the
// copies of the next task start while the current one is still being
// consumed, so short reductions (the down projection has 4 chunks) do not
// pay the pipeline fill per task.
//
// Records out of range (rows >= out, groups >= in/32) hold zero words, scales
// and biases, so they add exactly zero; no bounds checks in the inner loop.
// The pool is the counterpart of the reference's fixed-stride expert records
// (models/flashnext/slab_pack.py:1-25, expert_pool.py:1-22): expert e's
// records start at e * expert_stride.
#include "vx_async.cuh"
#include "vx_common.cuh"
#include "vx_launch.h"

namespace vx {

constexpr int kTiledThreads = 256;
constexpr int kTiledWarps = kTiledThreads / 32;
constexpr int kTiledStages = 4;

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

template <bool GATEUP, int MT, bool XMMA, int STAGES>
__global__ void __launch_bounds__(kTiledThreads, 2) gemv_tiled_kernel(const __grid_constant__ TiledArgs a) {
  constexpr int NP = GATEUP ? 2 : 1;
  constexpr int kRec = NP * MT * kTileRecordUnit;
  constexpr int kWBytes = NP * MT * 1024;
  constexpr int kXOff = kRec;                 // x: [i][b-lane g][16 B]
  constexpr int kXsOff = kRec + 512;          // sum(x) pairs [lane]
  constexpr int kStage = (kRec + 512 + (XMMA ? 0 : 256) + 127) & ~127;
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ __align__(8) uint64_t bars[kTiledWarps][STAGES];
  __shared__ __align__(16) uint32_t zero16[4];
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
  const bool blane = (g & 3) == c;   // carries token (g >> 2) on group c
  const int tb = g >> 2, ts = c >> 1;
  const int n_items = *a.n_items;
  const int total = n_items * a.tiles_per_item;
  const int nw = gridDim.x * kTiledWarps;
  const uint64_t pol = policy_evict_first();

  // ---- producer cursor: task ti, chunk ci ----
  int ti = blockIdx.x * kTiledWarps + warp, ci = 0;
  int inch = 0, iG = 0;   // chunks and groups of the task being issued
  const unsigned char* irec = nullptr;
  const uint16_t* ix = a.x;
  const float* ixs = a.xsum;
  bool ixv = false, ixsv = false;
  auto seek = [&]() {   // first valid task at or after ti
    for (; ti < total; ti += nw) {
      TiledTask k;
      if (!decode_task<MT>(a, ti, k)) continue;
      const int rb = k.row0 / (16 * MT);
      inch = (k.K + 127) >> 7;
      iG = k.K >> 5;
      irec = (k.sh ? a.rec_s : a.rec_b + int64_t(k.e) * a.stride_b) + int64_t(rb) * inch * kRec;
      ixv = blane && tb < k.cnt;
      ixsv = ts < k.cnt;
      int64_t rx = 0, rs = 0;
      if (ixv) rx = a.src_rows ? __ldg(a.src_rows + k.p0 + tb) : k.p0 + tb;
      if (!XMMA && ixsv) rs = a.src_rows ? __ldg(a.src_rows + k.p0 + ts) : k.p0 + ts;
      ix = a.x + rx * a.ldx + c * 32;
      if (!XMMA) ixs = a.xsum + rs * a.ldxs + 2 * (c & 1);
      return;
    }
  };
  int st_issue = 0, st_use = 0;
  uint32_t parity_bits = 0;   // bit s: parity expected next on stage s
  bool timed_out = false;
  auto issue = [&]() {
    const uint32_t st = ring + st_issue * kStage;
    if (lane == 0) {
      const uint32_t bar = bar0 + 8 * st_issue;
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      mbar_expect(bar, kRec);
      bulk_load(st, irec + int64_t(ci) * kRec, kRec, bar, pol);
    }
    const int nbytes = (ixv && 4 * ci + c < iG) ? 16 : 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) cp16_if(st + kXOff + (i * 8 + g) * 16, ix + ci * 128 + 8 * i, nbytes, blane);
    if (!XMMA) cp8(st + kXsOff + lane * 8, ixs + ci * 4, ixsv && 4 * ci + 2 * (c & 1) < iG);
    st_issue = st_issue == STAGES - 1 ? 0 : st_issue + 1;
    if (++ci == inch) {
      ci = 0;
      ti += nw;
      seek();
    }
  };

  seek();
#pragma unroll
  for (int s = 0; s < STAGES - 1; ++s) {
    if (ti < total) issue();
    cp_commit();
  }

  // ---- consumer: tasks in the same order ----
  for (int t = blockIdx.x * kTiledWarps + warp; t < total; t += nw) {
    TiledTask k;
    if (!decode_task<MT>(a, t, k)) continue;   // warp-uniform
    float acc[NP][MT][2];
#pragma unroll
    for (int p = 0; p < NP; ++p)
#pragma unroll
      for (int m = 0; m < MT; ++m) acc[p][m][0] = acc[p][m][1] = 0.f;

    const int nch = (k.K + 127) >> 7;
    for (int ch = 0; ch < nch; ++ch) {
      if (ti < total) issue();
      cp_commit();
      cp_wait<STAGES - 1>();
      const uint32_t st = ring + st_use * kStage;
      if (!mbar_wait(bar0 + 8 * st_use, (parity_bits >> st_use) & 1u)) timed_out = true;
      parity_bits ^= 1u << st_use;

      uint32_t bq[16];
      const uint32_t xa = blane ? st + kXOff + g * 16 : zaddr;
      const uint32_t xstep = blane ? 8 * 16 : 0;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint4 v = lds128(xa + i * xstep);
        bq[4 * i + 0] = v.x;
        bq[4 * i + 1] = v.y;
        bq[4 * i + 2] = v.z;
        bq[4 * i + 3] = v.w;
      }
      float xs0, xs1;
      if (XMMA) {
        float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int mm = 0; mm < 8; ++mm)
          mma16816(d, 0x3F803F80u, 0x3F803F80u, 0x3F803F80u, 0x3F803F80u, bq[2 * mm], bq[2 * mm + 1]);
        xs0 = d[0];
        xs1 = d[1];
      } else {
        const uint2 v = lds64(st + kXsOff + lane * 8);
        xs0 = __uint_as_float(v.x);
        xs1 = __uint_as_float(v.y);
      }
#pragma unroll
      for (int p = 0; p < NP; ++p) {
#pragma unroll
        for (int m = 0; m < MT; ++m) {
          const uint32_t wrow = st + (p * MT + m) * 1024 + lane * 16;
          const uint4 wg = lds128(wrow), w8 = lds128(wrow + 512);
          const uint32_t ag[4] = {wg.x, wg.y, wg.z, wg.w};
          const uint32_t a8[4] = {w8.x, w8.y, w8.z, w8.w};
          float d[4] = {0.f, 0.f, 0.f, 0.f}, e2[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int mm = 0; mm < 8; mm += 2) {
            const int wi = mm >> 1;
            mma16816(d, nib_pair128(ag[wi]), nib_pair128(a8[wi]), nib_pair128(ag[wi] >> 4),
                     nib_pair128(a8[wi] >> 4), bq[2 * mm], bq[2 * mm + 1]);
            mma16816(e2, nib_pair128(ag[wi] >> 8), nib_pair128(a8[wi] >> 8),
                     nib_pair128(ag[wi] >> 12), nib_pair128(a8[wi] >> 12), bq[2 * mm + 2],
                     bq[2 * mm + 3]);
          }
#pragma unroll
          for (int i = 0; i < 4; ++i) d[i] += e2[i];
          const uint4 sb = lds128(st + kWBytes + (p * MT + m) * 256 + (g * 2 + (c & 1)) * 16);
          const uint32_t sw[4] = {sb.x, sb.y, sb.z, sb.w};
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const float s0 = __uint_as_float(sw[2 * h] << 16);
            const float s1 = __uint_as_float(sw[2 * h] & 0xFFFF0000u);
            const float b0 = __uint_as_float(sw[2 * h + 1] << 16);
            const float b1 = __uint_as_float(sw[2 * h + 1] & 0xFFFF0000u);
            // bias - 128*scale: the lop3 operands carry q + 128.
            const float c0 = fmaf(-128.f, s0, b0);
            const float c1 = fmaf(-128.f, s1, b1);
            float v = acc[p][m][h];
            v = fmaf(s0, d[2 * h], v);
            v = fmaf(c0, xs0, v);
            v = fmaf(s1, d[2 * h + 1], v);
            v = fmaf(c1, xs1, v);
            acc[p][m][h] = v;
          }
        }
      }
      __syncwarp();   // the stage is read out before the warp refills it
      st_use = st_use == STAGES - 1 ? 0 : st_use + 1;
    }

#pragma unroll
    for (int p = 0; p < NP; ++p)
#pragma unroll
      for (int m = 0; m < MT; ++m)
#pragma unroll
        for (int h = 0; h < 2; ++h) acc[p][m][h] += __shfl_xor_sync(0xFFFFFFFFu, acc[p][m][h], 1);
    const int tok = c >> 1;
    if ((c & 1) == 0 && tok < k.cnt) {
      const int pos = k.p0 + tok;
      const int64_t dst = a.dst_rows ? __ldg(a.dst_rows + pos) : pos;
#pragma unroll
      for (int m = 0; m < MT; ++m)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int row = k.row0 + 16 * m + g + 8 * h;
          if (row >= k.N) continue;
          if (GATEUP) {
            const float v = silu_mul_bf16(bf16r(acc[0][m][h]), bf16r(acc[NP - 1][m][h]));
            a.out[dst * a.ldo + b_order_col(row)] = f32_to_bf16(v);
          } else {
            a.out[dst * a.ldo + row] = f32_to_bf16(acc[0][m][h]);
          }
        }
    }
  }
  cp_wait<0>();
  if (timed_out && a.err) atomicOr(a.err, 0x100);
}

// ---- pool packing -----------------------------------------------------------

// One thread per 16-byte unit of the pool.  a: first (or only) projection,
// b: second projection of a gate/up pair.
__global__ void tile_pack_kernel(vx_q4 a, vx_q4 b, int NP, int MT, int RB, int nch, uint4* out,
                                 int64_t units) {
  const int per_rec = NP * MT * (kTileRecordUnit / 16);
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

int64_t tile_pool_bytes(int64_t experts, int out, int in, int nproj, int tile_rows) {
  const int64_t RB = (out + tile_rows - 1) / tile_rows;
  const int64_t nch = (in + 127) / 128;
  return experts * RB * nch * int64_t(nproj) * (tile_rows / 16) * kTileRecordUnit;
}

cudaError_t launch_tile_pack(const vx_q4& a, const vx_q4& b, int nproj, int tile_rows, void* out,
                             cudaStream_t st) {
  const int MT = tile_rows / 16;
  const int RB = (a.out + tile_rows - 1) / tile_rows;
  const int nch = (a.in + 127) / 128;
  const int64_t units = tile_pool_bytes(a.experts, a.out, a.in, nproj, tile_rows) / 16;
  if (units == 0) return cudaSuccess;
  int64_t blocks = (units + 255) / 256;
  if (blocks > int64_t(sm_count()) * 32) blocks = int64_t(sm_count()) * 32;
  tile_pack_kernel<<<int(blocks), 256, 0, st>>>(a, nproj == 2 ? b : a, nproj, MT, RB, nch,
                                                static_cast<uint4*>(out), units);
  return cudaGetLastError();
}

// ---- launcher ----------------------------------------------------------------

template <bool GATEUP, int MT, bool XMMA>
static cudaError_t launch_tiled_t(TiledArgs a, int max_items, int max_out, cudaStream_t st) {
  constexpr int NP = GATEUP ? 2 : 1;
  constexpr int kRec = NP * MT * kTileRecordUnit;
  constexpr int kStage = (kRec + 512 + (XMMA ? 0 : 256) + 127) & ~127;
  a.tiles_per_item = (max_out + 16 * MT - 1) / (16 * MT);
  const size_t smem = size_t(kTiledWarps) * kTiledStages * kStage;
  auto kern = gemv_tiled_kernel<GATEUP, MT, XMMA, kTiledStages>;
  cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (err != cudaSuccess) return err;
  const int64_t warps = int64_t(max_items) * a.tiles_per_item;
  const int64_t cap = int64_t(sm_count()) * 2;   // two resident CTAs per SM, persistent
  int64_t grid = (warps + kTiledWarps - 1) / kTiledWarps;
  if (grid > cap) grid = cap;
  if (grid <= 0) return cudaSuccess;
  kern<<<int(grid), kTiledThreads, smem, st>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_gemv_tiled(bool gateup, int tile_rows, const TiledArgs& a, int max_items,
                              int max_out, cudaStream_t st) {
  const bool xmma = a.xsum == nullptr;
  if (gateup) {
    if (tile_rows != 16) return cudaErrorInvalidValue;
    return xmma ? launch_tiled_t<true, 1, true>(a, max_items, max_out, st)
                : launch_tiled_t<true, 1, false>(a, max_items, max_out, st);
  }
  if (tile_rows == 32)
    return xmma ? launch_tiled_t<false, 2, true>(a, max_items, max_out, st)
                : launch_tiled_t<false, 2, false>(a, max_items, max_out, st);
  if (tile_rows == 16)
    return xmma ? launch_tiled_t<false, 1, true>(a, max_items, max_out, st)
                : launch_tiled_t<false, 1, false>(a, max_items, max_out, st);
  return cudaErrorInvalidValue;
}

}  // namespace vx
