// Grouped Q4 GEMV on the tensor pipe (sm_100a, mma.sync m16n8k16 bf16).
//
// Regime: few tokens per expert (decode, batched decode).  Work unit = one
// warp x (item, block of 16*MT output rows); an item is an expert with up to
// kItemChunk expert-sorted tokens (built by the permute kernel).  Every warp
// streams its rows over the whole input width through its own 3-stage
// cp.async ring in shared memory (weights, scales and activations), so the
// bytes in flight do not cost registers and no block synchronisation is
// needed: each lane only reads back what it copied itself.
//
// Layout trick ("block-diagonal B").  Lane (g = lane/4, c = lane%4) copies 16
// bytes of row g (and row g+8): words 4c..4c+3 of a 128-input chunk, i.e. the
// whole quant group c of that chunk.  Each nibble becomes an exact bf16 via
// lop3 (0x4300 | q = 128+q) and a bf16x2 subtract of 128.  Within one
// m16n8k16 MMA lane c supplies four inputs of its own group, so one MMA mixes
// four groups along k.  B is block-diagonal: column n = 4*tok + grp holds
// token tok's x only on the k positions of group grp and zero elsewhere, so
// D[row][4*tok + grp] is the per-group partial sum(q*x) of that row - the
// quantity MLX's qmv scales by the group's scale (models/flashnext/
// metal_runtime.py:1014-1029).  Eight MMAs cover a chunk of 4 groups for two
// tokens; an MMA with A = ones over the same B yields sum(x) per group.  The
// epilogue adds scale*sum(q*x) + bias*sum(x) per group in float32, and the
// two lanes holding a row's group halves meet in one shuffle.  An item's
// token pairs share one sweep over the weights: every unpacked A fragment
// feeds one MMA per pair.
#include "vx_common.cuh"
#include "vx_launch.h"

namespace vx {

constexpr int kMmaThreads = 256;
constexpr int kStages = 3;
constexpr int kPairs = kItemChunk / 2;

VX_DEVICE uint32_t nib_pair(uint32_t w_shifted) {
  // {128 + (w & 15), 128 + ((w >> 16) & 15)} as bf16x2, then minus 128: exact.
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(w_shifted), "r"(0x000F000Fu), "r"(0x43004300u));
  uint32_t out;
  asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(out) : "r"(r), "r"(0x3F803F80u), "r"(0xC300C300u));
  return out;
}

VX_DEVICE uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// 16/4-byte async copies; src_bytes = 0 writes zeros without reading.
VX_DEVICE void cp16(void* dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src),
               "r"(valid ? 16 : 0)
               : "memory");
}
VX_DEVICE void cp4(void* dst, const void* src, bool valid) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(smem_u32(dst)), "l"(src),
               "r"(valid ? 4 : 0)
               : "memory");
}
VX_DEVICE void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
VX_DEVICE void cp_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// Per-warp stage, in 16-byte units.
template <int NP, int MT>
struct StageLayout {
  static constexpr int kW = NP * MT * 2 * 32;            // weights [p][m][h][lane]
  static constexpr int kS = NP * MT * 2 * 32 / 2;        // scale+bias pairs, 8 B each
  static constexpr int kX = kPairs * 8 * 4;              // x: [pair][b-lane g][4]
  static constexpr int kTotal = kW + kS + kX;
};

template <bool GATEUP, int MT>
__global__ void __launch_bounds__(kMmaThreads, 2) gemv_mma_kernel(MmaArgs a) {
  constexpr int NP = GATEUP ? 2 : 1;
  using L = StageLayout<NP, MT>;
  extern __shared__ uint4 smem4[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;
  uint4* ring = smem4 + warp * kStages * L::kTotal;
  const int n_items = *a.n_items;
  const int total = n_items * a.tiles_per_item;
  const int nw = gridDim.x * (kMmaThreads / 32);
  for (int t = blockIdx.x * (kMmaThreads / 32) + warp; t < total; t += nw) {
    const int item = t / a.tiles_per_item, rb = t - item * a.tiles_per_item;
    const int e = __ldg(a.items + 3 * item), p0 = __ldg(a.items + 3 * item + 1);
    const int cnt = __ldg(a.items + 3 * item + 2);
    const bool sh = e == a.E;
    Q4Ptr pp[NP];
    const vx_q4& B0 = sh ? a.s0 : a.b0;
    pp[0] = q4_expert(B0, sh ? 0 : e);
    if (GATEUP) pp[NP - 1] = q4_expert(sh ? a.s1 : a.b1, sh ? 0 : e);
    const int N = B0.out, K = B0.in, KW = K >> 3, G = K >> 5;
    const bool even_g = (G & 1) == 0;
    const int nch = (K + 127) >> 7;
    const int row0 = rb * 16 * MT;
    if (row0 >= N) continue;  // warp-uniform
    const int npairs = (cnt + 1) >> 1;

    int rows[MT][2];
    bool rv[MT][2];
#pragma unroll
    for (int m = 0; m < MT; ++m)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        rows[m][h] = row0 + 16 * m + g + 8 * h;
        rv[m][h] = rows[m][h] < N;
      }
    // B lanes: (g & 3) == c carries token 2*pair + (g >> 2) on group c.
    const bool blane = (g & 3) == c;
    const uint16_t* xrow[kPairs];
#pragma unroll
    for (int q = 0; q < kPairs; ++q) {
      const int tok = 2 * q + (g >> 2);
      xrow[q] = nullptr;
      if (blane && tok < cnt) {
        const int pos = p0 + tok;
        const int64_t r = a.src_rows ? __ldg(a.src_rows + pos) : pos;
        xrow[q] = a.x + r * a.ldx;
      }
    }

    auto issue = [&](int ch) {
      uint4* st = ring + (ch % kStages) * L::kTotal;
      const int grp = 4 * ch + c;
#pragma unroll
      for (int p = 0; p < NP; ++p)
#pragma unroll
        for (int m = 0; m < MT; ++m)
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const bool ok = rv[m][h] && grp < G;
            const uint32_t* src = ok ? pp[p].w + int64_t(rows[m][h]) * KW + grp * 4 : pp[p].w;
            cp16(st + ((p * MT + m) * 2 + h) * 32 + lane, src, ok);
          }
      if (even_g) {
        const int gA = 4 * ch + 2 * (c & 1);
        uint32_t* sp = reinterpret_cast<uint32_t*>(st + L::kW);
#pragma unroll
        for (int p = 0; p < NP; ++p)
#pragma unroll
          for (int m = 0; m < MT; ++m)
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const bool ok = rv[m][h] && gA < G;
              const int64_t mi = ok ? int64_t(rows[m][h]) * G + gA : 0;
              const int slot = ((p * MT + m) * 2 + h) * 32 + lane;
              cp4(sp + 2 * slot, pp[p].s + mi, ok);
              cp4(sp + 2 * slot + 1, pp[p].b + mi, ok);
            }
      }
      if (blane) {
        uint4* xp = st + L::kW + L::kS;
#pragma unroll
        for (int q = 0; q < kPairs; ++q) {
          const bool ok = xrow[q] != nullptr && grp < G;
          const uint16_t* src = ok ? xrow[q] + grp * 32 : a.x;
#pragma unroll
          for (int i = 0; i < 4; ++i) cp16(xp + (q * 8 + g) * 4 + i, src + 8 * i, ok);
        }
      }
    };

    float acc[kPairs][NP][MT][2];
#pragma unroll
    for (int q = 0; q < kPairs; ++q)
#pragma unroll
      for (int p = 0; p < NP; ++p)
#pragma unroll
        for (int m = 0; m < MT; ++m) acc[q][p][m][0] = acc[q][p][m][1] = 0.f;

#pragma unroll
    for (int s = 0; s < kStages - 1; ++s) {
      if (s < nch) issue(s);
      cp_commit();
    }
    for (int ch = 0; ch < nch; ++ch) {
      if (ch + kStages - 1 < nch) issue(ch + kStages - 1);
      cp_commit();
      cp_wait<kStages - 1>();
      const uint4* st = ring + (ch % kStages) * L::kTotal;
      // B fragments and sum(x) per pair.
      uint32_t bq[kPairs][16];
      float xs[kPairs][4];
#pragma unroll
      for (int q = 0; q < kPairs; ++q) {
        if (q < npairs && blane) {
          const uint4* xp = st + L::kW + L::kS + (q * 8 + g) * 4;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const uint4 v = xp[i];
            bq[q][4 * i + 0] = prmt(v.x, v.z, 0x5410);   // (x0, x4)
            bq[q][4 * i + 1] = prmt(v.x, v.z, 0x7632);   // (x1, x5)
            bq[q][4 * i + 2] = prmt(v.y, v.w, 0x5410);   // (x2, x6)
            bq[q][4 * i + 3] = prmt(v.y, v.w, 0x7632);   // (x3, x7)
          }
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i) bq[q][i] = 0u;
        }
        xs[q][0] = xs[q][1] = xs[q][2] = xs[q][3] = 0.f;
        if (q < npairs) {
#pragma unroll
          for (int mm = 0; mm < 8; ++mm)
            mma16816(xs[q], 0x3F803F80u, 0x3F803F80u, 0x3F803F80u, 0x3F803F80u, bq[q][2 * mm],
                     bq[q][2 * mm + 1]);
        }
      }
      const int gA = 4 * ch + 2 * (c & 1);   // groups of D columns 2c, 2c+1
#pragma unroll
      for (int p = 0; p < NP; ++p) {
#pragma unroll
        for (int m = 0; m < MT; ++m) {
          const uint4 wg = st[((p * MT + m) * 2 + 0) * 32 + lane];
          const uint4 w8 = st[((p * MT + m) * 2 + 1) * 32 + lane];
          const uint32_t ag[4] = {wg.x, wg.y, wg.z, wg.w};
          const uint32_t a8[4] = {w8.x, w8.y, w8.z, w8.w};
          float d[kPairs][4];
#pragma unroll
          for (int q = 0; q < kPairs; ++q) d[q][0] = d[q][1] = d[q][2] = d[q][3] = 0.f;
#pragma unroll
          for (int mm = 0; mm < 8; ++mm) {
            const int wi = mm >> 1;
            const int s = (mm & 1) ? 8 : 0;
            const uint32_t a0 = nib_pair(ag[wi] >> s), a1 = nib_pair(a8[wi] >> s);
            const uint32_t a2 = nib_pair(ag[wi] >> (s + 4)), a3 = nib_pair(a8[wi] >> (s + 4));
            mma16816(d[0], a0, a1, a2, a3, bq[0][2 * mm], bq[0][2 * mm + 1]);
#pragma unroll
            for (int q = 1; q < kPairs; ++q)
              if (q < npairs) mma16816(d[q], a0, a1, a2, a3, bq[q][2 * mm], bq[q][2 * mm + 1]);
          }
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            if (!rv[m][h] || gA >= G) continue;
            float s0, s1, b0, b1;
            if (even_g) {
              const uint2 sb = reinterpret_cast<const uint2*>(st + L::kW)[((p * MT + m) * 2 + h) * 32 + lane];
              s0 = __uint_as_float(sb.x << 16);
              s1 = __uint_as_float(sb.x & 0xFFFF0000u);
              b0 = __uint_as_float(sb.y << 16);
              b1 = __uint_as_float(sb.y & 0xFFFF0000u);
            } else {
              const int64_t mi = int64_t(rows[m][h]) * G + gA;
              const bool two = gA + 1 < G;
              s0 = bf16_to_f32(pp[p].s[mi]);
              b0 = bf16_to_f32(pp[p].b[mi]);
              s1 = two ? bf16_to_f32(pp[p].s[mi + 1]) : 0.f;
              b1 = two ? bf16_to_f32(pp[p].b[mi + 1]) : 0.f;
            }
#pragma unroll
            for (int q = 0; q < kPairs; ++q) {
              float v = acc[q][p][m][h];
              v += fmaf(s0, d[q][2 * h], b0 * xs[q][0]);
              v += fmaf(s1, d[q][2 * h + 1], b1 * xs[q][1]);
              acc[q][p][m][h] = v;
            }
          }
        }
      }
    }
    cp_wait<0>();
    // lanes c and c^1 hold the two group halves of the same (row, token)
#pragma unroll
    for (int q = 0; q < kPairs; ++q) {
#pragma unroll
      for (int p = 0; p < NP; ++p)
#pragma unroll
        for (int m = 0; m < MT; ++m)
#pragma unroll
          for (int h = 0; h < 2; ++h)
            acc[q][p][m][h] += __shfl_xor_sync(0xFFFFFFFFu, acc[q][p][m][h], 1);
      const int tok = 2 * q + (c >> 1);
      if ((c & 1) == 0 && tok < cnt) {
        const int pos = p0 + tok;
        const int64_t dst = a.dst_rows ? __ldg(a.dst_rows + pos) : pos;
#pragma unroll
        for (int m = 0; m < MT; ++m)
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            if (!rv[m][h]) continue;
            float v;
            if (GATEUP) v = silu_mul_bf16(bf16r(acc[q][0][m][h]), bf16r(acc[q][NP - 1][m][h]));
            else v = acc[q][0][m][h];
            a.out[dst * a.ldo + rows[m][h]] = f32_to_bf16(v);
          }
      }
    }
  }
}

template <bool GATEUP, int MT>
static cudaError_t launch_mma_t(MmaArgs a, int max_items, int max_out, cudaStream_t st) {
  constexpr int NP = GATEUP ? 2 : 1;
  a.tiles_per_item = (max_out + 16 * MT - 1) / (16 * MT);
  const size_t smem = size_t(kMmaThreads / 32) * kStages * StageLayout<NP, MT>::kTotal * sizeof(uint4);
  auto kern = gemv_mma_kernel<GATEUP, MT>;
  cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (err != cudaSuccess) return err;
  const int64_t warps = int64_t(max_items) * a.tiles_per_item;
  const int64_t cap = int64_t(sm_count()) * 2;  // two resident CTAs per SM, persistent
  int64_t grid = (warps + 7) / 8;
  if (grid > cap) grid = cap;
  if (grid <= 0) return cudaSuccess;
  kern<<<int(grid), kMmaThreads, smem, st>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_gemv_mma(bool gateup, const MmaArgs& a, int max_items, int max_out,
                            cudaStream_t st) {
  // gate/up holds two projections per row block: one m-tile each.  The down
  // projection takes 32-row tiles when there is plenty of work.
  if (gateup) return launch_mma_t<true, 1>(a, max_items, max_out, st);
  const int64_t rows_work = int64_t(max_items) * max_out;
  const bool small = rows_work < int64_t(sm_count()) * 16 * 32;
  return small ? launch_mma_t<false, 1>(a, max_items, max_out, st)
               : launch_mma_t<false, 2>(a, max_items, max_out, st);
}

}  // namespace vx
