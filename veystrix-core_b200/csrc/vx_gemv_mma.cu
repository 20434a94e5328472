// Grouped Q4 GEMV on the tensor pipe (sm_100a, mma.sync m16n8k16 bf16).
//
// Regime: few tokens per expert (decode, batched decode).  Work unit = one
// warp x (item, block of 16*MT output rows); an item is an expert with up to
// kItemChunk expert-sorted tokens (built by the permute kernel).  The warp
// streams its rows over the whole input width with 128-bit loads straight
// from global memory - no shared memory, no block synchronisation - so every
// warp keeps its own loads in flight.
//
// Layout trick ("block-diagonal B").  Lane (g = lane/4, c = lane%4) loads 16
// bytes of row g (and row g+8): words 4c..4c+3 of a 128-input chunk, i.e. the
// whole quant group c of that chunk.  Each nibble becomes an exact bf16 via
// lop3 (0x4300 | q = 128+q) and a bf16x2 subtract of 128.  Within one
// m16n8k16 MMA lane c supplies four inputs of its own group, so one MMA
// mixes four groups along k.  B is block-diagonal: column n = 4*tok + grp
// holds token tok's x only on the k positions of group grp, zero elsewhere,
// so D[row][4*tok + grp] is the per-group partial sum(q*x) of that row - the
// quantity MLX's qmv scales by the group's scale (models/flashnext/
// metal_runtime.py:1014-1029).  Eight MMAs cover a chunk of 4 groups for two
// tokens; an MMA with A = ones over the same B yields sum(x) per group.  The
// epilogue adds scale*sum(q*x) + bias*sum(x) per group in float32 and the
// two lanes holding a row's group halves meet in one shuffle.
#include "vx_common.cuh"
#include "vx_launch.h"

namespace vx {

constexpr int kMmaThreads = 256;

VX_DEVICE uint32_t nib_pair(uint32_t w_shifted) {
  // {128 + (w & 15), 128 + ((w >> 16) & 15)} as bf16x2, then minus 128: exact.
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(w_shifted), "r"(0x000F000Fu), "r"(0x43004300u));
  uint32_t out;
  asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(out) : "r"(r), "r"(0x3F803F80u), "r"(0xC300C300u));
  return out;
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

VX_DEVICE uint4 ldg_nc(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// D += A(row g / g+8 words) x B for the 8 MMAs of one 128-input chunk.
VX_DEVICE void chunk_mma(float (&d)[4], const uint4& wg, const uint4& w8, const uint32_t (&bq)[16]) {
  const uint32_t ag[4] = {wg.x, wg.y, wg.z, wg.w};
  const uint32_t a8[4] = {w8.x, w8.y, w8.z, w8.w};
#pragma unroll
  for (int m = 0; m < 8; ++m) {
    const int wi = m >> 1;
    const int s = (m & 1) ? 8 : 0;
    mma16816(d, nib_pair(ag[wi] >> s), nib_pair(a8[wi] >> s), nib_pair(ag[wi] >> (s + 4)),
             nib_pair(a8[wi] >> (s + 4)), bq[2 * m], bq[2 * m + 1]);
  }
}

template <bool GATEUP, int MT>
__global__ void __launch_bounds__(kMmaThreads, 2) gemv_mma_kernel(MmaArgs a) {
  constexpr int NP = GATEUP ? 2 : 1;
  const int lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;
  const int n_items = *a.n_items;
  const int total = n_items * a.tiles_per_item;
  const int nw = gridDim.x * (kMmaThreads / 32);
  for (int t = blockIdx.x * (kMmaThreads / 32) + (threadIdx.x >> 5); t < total; t += nw) {
    const int item = t / a.tiles_per_item, rb = t - item * a.tiles_per_item;
    const int e = __ldg(a.items + 3 * item), p0 = __ldg(a.items + 3 * item + 1);
    const int cnt = __ldg(a.items + 3 * item + 2);
    const bool sh = e == a.E;
    Q4Ptr pp[NP];
    const vx_q4& B0 = sh ? a.s0 : a.b0;
    pp[0] = q4_expert(B0, sh ? 0 : e);
    if (GATEUP) pp[NP - 1] = q4_expert(sh ? a.s1 : a.b1, sh ? 0 : e);
    const int N = B0.out, K = B0.in, KW = K >> 3, G = K >> 5;
    const int nch = (K + 127) >> 7;
    const int row0 = rb * 16 * MT;
    if (row0 >= N) continue;

    int rows[MT][2];
    bool rv[MT][2];
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      rows[m][0] = row0 + 16 * m + g;
      rows[m][1] = row0 + 16 * m + g + 8;
      rv[m][0] = rows[m][0] < N;
      rv[m][1] = rows[m][1] < N;
    }

    for (int pass = 0; pass < cnt; pass += 2) {
      // B lane role: lanes with (g & 3) == c carry token (g >> 2) of this
      // pass on group c of each chunk; all other lanes hold zeros.
      const int tb = g >> 2;
      const bool bl = ((g & 3) == c) && (pass + tb < cnt);
      const uint16_t* xrow = nullptr;
      if (bl) {
        const int pos = p0 + pass + tb;
        const int64_t r = a.src_rows ? __ldg(a.src_rows + pos) : pos;
        xrow = a.x + r * a.ldx;
      }
      float acc[NP][MT][2];
#pragma unroll
      for (int p = 0; p < NP; ++p)
#pragma unroll
        for (int m = 0; m < MT; ++m) acc[p][m][0] = acc[p][m][1] = 0.f;

      uint4 wcur[NP][MT][2], wnext[NP][MT][2];
      auto load_chunk = [&](int ch, uint4 (&w)[NP][MT][2]) {
        const int grp = 4 * ch + c;
#pragma unroll
        for (int p = 0; p < NP; ++p)
#pragma unroll
          for (int m = 0; m < MT; ++m)
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              if (rv[m][h] && grp < G)
                w[p][m][h] = ldg_nc(pp[p].w + int64_t(rows[m][h]) * KW + grp * 4);
              else
                w[p][m][h] = make_uint4(0, 0, 0, 0);
            }
      };
      load_chunk(0, wcur);
      for (int ch = 0; ch < nch; ++ch) {
        if (ch + 1 < nch) load_chunk(ch + 1, wnext);
        // B fragments: 32 x values of (token tb, group c of this chunk).
        uint32_t bq[16];
        if (bl && 4 * ch + c < G) {
          const uint4* xp = reinterpret_cast<const uint4*>(xrow + (4 * ch + c) * 32);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const uint4 v = __ldg(xp + q);
            bq[4 * q + 0] = prmt(v.x, v.z, 0x5410);   // (x0, x4)
            bq[4 * q + 1] = prmt(v.x, v.z, 0x7632);   // (x1, x5)
            bq[4 * q + 2] = prmt(v.y, v.w, 0x5410);   // (x2, x6)
            bq[4 * q + 3] = prmt(v.y, v.w, 0x7632);   // (x3, x7)
          }
        } else {
#pragma unroll
          for (int q = 0; q < 16; ++q) bq[q] = 0u;
        }
        // sum(x) per (token, group) in the D layout: A = ones.
        float xs[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int m = 0; m < 8; ++m)
          mma16816(xs, 0x3F803F80u, 0x3F803F80u, 0x3F803F80u, 0x3F803F80u, bq[2 * m], bq[2 * m + 1]);
        const int gA = 4 * ch + 2 * (c & 1);   // groups of D columns 2c, 2c+1
#pragma unroll
        for (int p = 0; p < NP; ++p) {
#pragma unroll
          for (int m = 0; m < MT; ++m) {
            float d[4] = {0.f, 0.f, 0.f, 0.f};
            chunk_mma(d, wcur[p][m][0], wcur[p][m][1], bq);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              if (!rv[m][h] || gA >= G) continue;
              const int64_t mi = int64_t(rows[m][h]) * G + gA;
              float s0, s1, b0, b1;
              // paired 4-byte loads need an even group count (alignment)
              if (gA + 1 < G && (G & 1) == 0) {
                const uint32_t sv = __ldg(reinterpret_cast<const uint32_t*>(pp[p].s + mi));
                const uint32_t bv = __ldg(reinterpret_cast<const uint32_t*>(pp[p].b + mi));
                s0 = __uint_as_float(sv << 16);
                s1 = __uint_as_float(sv & 0xFFFF0000u);
                b0 = __uint_as_float(bv << 16);
                b1 = __uint_as_float(bv & 0xFFFF0000u);
              } else {
                s0 = bf16_to_f32(pp[p].s[mi]);
                b0 = bf16_to_f32(pp[p].b[mi]);
                const bool two = gA + 1 < G;
                s1 = two ? bf16_to_f32(pp[p].s[mi + 1]) : 0.f;
                b1 = two ? bf16_to_f32(pp[p].b[mi + 1]) : 0.f;
              }
              float v = acc[p][m][h];
              v += fmaf(s0, d[2 * h], b0 * xs[0]);
              v += fmaf(s1, d[2 * h + 1], b1 * xs[1]);
              acc[p][m][h] = v;
            }
          }
        }
        if (ch + 1 < nch) {
#pragma unroll
          for (int p = 0; p < NP; ++p)
#pragma unroll
            for (int m = 0; m < MT; ++m) {
              wcur[p][m][0] = wnext[p][m][0];
              wcur[p][m][1] = wnext[p][m][1];
            }
        }
      }
      // lanes c and c^1 hold the two group halves of the same (row, token)
#pragma unroll
      for (int p = 0; p < NP; ++p)
#pragma unroll
        for (int m = 0; m < MT; ++m)
#pragma unroll
          for (int h = 0; h < 2; ++h) acc[p][m][h] += __shfl_xor_sync(0xFFFFFFFFu, acc[p][m][h], 1);
      const int tok = pass + (c >> 1);
      if ((c & 1) == 0 && tok < cnt) {
        const int pos = p0 + tok;
        const int64_t dst = a.dst_rows ? __ldg(a.dst_rows + pos) : pos;
#pragma unroll
        for (int m = 0; m < MT; ++m)
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            if (!rv[m][h]) continue;
            float v;
            if (GATEUP) v = silu_mul_bf16(bf16r(acc[0][m][h]), bf16r(acc[NP - 1][m][h]));
            else v = acc[0][m][h];
            a.out[dst * a.ldo + rows[m][h]] = f32_to_bf16(v);
          }
      }
    }
  }
}

template <bool GATEUP, int MT>
static cudaError_t launch_mma_t(MmaArgs a, int max_items, int max_out, cudaStream_t st) {
  a.tiles_per_item = (max_out + 16 * MT - 1) / (16 * MT);
  const int64_t warps = int64_t(max_items) * a.tiles_per_item;
  const int64_t cap = int64_t(sm_count()) * 8;  // CTAs: 8 warps each, ~8 CTAs per SM
  int64_t grid = (warps + 7) / 8;
  if (grid > cap) grid = cap;
  if (grid <= 0) return cudaSuccess;
  gemv_mma_kernel<GATEUP, MT><<<int(grid), kMmaThreads, 0, st>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_gemv_mma(bool gateup, const MmaArgs& a, int max_items, int max_out,
                            cudaStream_t st) {
  // Fewer, longer warp tiles when there is plenty of work; 16-row tiles when
  // the batch is small so that every SM gets warps.
  const int64_t rows_work = int64_t(max_items) * max_out;
  const bool small = rows_work < int64_t(sm_count()) * 8 * 32;
  // gate/up holds two projections per row block: one m-tile each keeps it
  // within the 128-register budget of two CTAs per SM.
  if (gateup) return launch_mma_t<true, 1>(a, max_items, max_out, st);
  return small ? launch_mma_t<false, 1>(a, max_items, max_out, st)
               : launch_mma_t<false, 2>(a, max_items, max_out, st);
}

}  // namespace vx
