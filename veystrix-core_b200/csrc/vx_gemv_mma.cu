// Grouped Q4 GEMV on the tensor pipe (sm_100a, mma.sync m16n8k16 bf16).
//
// Regime: few tokens per expert (decode, batched decode).  Work unit = one
// warp x (item, block of 16*MT output rows); an item is an expert with up to
// two expert-sorted tokens (built by the permute kernel).  Each warp streams
// its rows over the whole input width through its own 3-stage pipeline in
// shared memory: one lane issues a 2-D TMA copy per projection per
// 128-input chunk (16*MT rows x 64 bytes, completed on an mbarrier), and the
// small operands - activations, their per-group sums, the group
// scales/biases - ride cp.async copies into the same stage.  No block
// synchronisation: the warp's own mbarriers and async-copy groups order it.
//
// Layout trick ("block-diagonal B").  Lane (g = lane/4, c = lane%4) reads 16
// bytes of row g (and row g+8): words 4c..4c+3 of the chunk, i.e. the whole
// quant group c.  A nibble q becomes the exact bf16 128+q through one lop3
// with 0x4300.  Within one m16n8k16 MMA lane c supplies four inputs of its
// own group, so one MMA mixes four groups along k.  B is block-diagonal:
// column n = 4*tok + grp holds token tok's x only on the k positions of
// group grp, so D[row][4*tok + grp] = sum((128+q)*x) over that group.  The
// epilogue applies MLX's qmv formula per group (models/flashnext/
// metal_runtime.py:1014-1029),
//     scale*sum(q*x) + bias*sum(x) = scale*D + (bias - 128*scale)*sum(x),
// in float32; the two lanes holding a row's group halves meet in one shuffle.
//
// Activations arrive in "B order" (within each 8-input block the words hold
// the pairs (0,4) (1,5) (2,6) (3,7)), so a B lane's 16-byte loads are its
// MMA fragments as they stand; sum(x) per group comes from a precomputed
// table (gate/up, gather_qmm) or from an MMA with A = ones over the same B
// (down, whose input h this kernel writes itself).
#include <cudaTypedefs.h>

#include "vx_async.cuh"
#include "vx_common.cuh"
#include "vx_launch.h"

namespace vx {

constexpr int kMmaThreads = 256;
constexpr int kWarps = kMmaThreads / 32;
constexpr int kStages = 3;
// One pipeline stage of one warp, bytes (multiples of 128).
template <int NP, int MT, bool XMMA>
struct Stage {
  static constexpr int kWRows = 16 * MT;
  static constexpr int kW = NP * kWRows * 64;            // TMA boxes [p][row][64 B]
  static constexpr int kS = NP * MT * 32 * 16;           // scales [p][m][lane]{s_g b_g s_g8 b_g8}
  static constexpr int kX = 4 * 8 * 16;                  // x: [i][b-lane g][16 B]
  static constexpr int kXS = XMMA ? 0 : 32 * 8;          // sum(x) pairs [lane]
  static constexpr int kRaw = kW + kS + kX + kXS;
  static constexpr int kBytes = (kRaw + 127) & ~127;
};

template <bool GATEUP, int MT, bool XMMA, bool EVEN>
__global__ void __launch_bounds__(kMmaThreads, 2) gemv_mma_kernel(const __grid_constant__ MmaArgs a) {
  chain_wait();
  constexpr int NP = GATEUP ? 2 : 1;
  using S = Stage<NP, MT, XMMA>;
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ __align__(8) uint64_t bars[kWarps][kStages];
  __shared__ __align__(16) uint32_t zero16[4];   // B operand of the non-B lanes
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, c = lane & 3;
  if (threadIdx.x < 4) zero16[threadIdx.x] = 0u;
  if (lane == 0)
    for (int s = 0; s < kStages; ++s) mbar_init(smem_u32(&bars[warp][s]));
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  __syncthreads();
  const uint32_t ring = smem_u32(smem) + warp * kStages * S::kBytes;
  const uint32_t bar0 = smem_u32(&bars[warp][0]);
  const uint32_t zaddr = smem_u32(zero16);
  const bool blane = (g & 3) == c;   // carries token (g >> 2) on group c
  const int n_items = *a.n_items;
  const int total = n_items * a.tiles_per_item;
  const int nw = gridDim.x * kWarps;
  // Ring position of the next chunk to issue / consume, and the mbarrier
  // phase parity of the consumed stage.
  int st_issue = 0, st_use = 0;
  uint32_t parity_bits = 0;          // bit s: parity expected next on stage s
  bool timed_out = false;

  for (int t = blockIdx.x * kWarps + warp; t < total; t += nw) {
    const int item = t / a.tiles_per_item, rb = t - item * a.tiles_per_item;
    const int e = __ldg(a.items + 3 * item), p0 = __ldg(a.items + 3 * item + 1);
    const int cnt = __ldg(a.items + 3 * item + 2);
    const bool sh = e == a.E;
    const vx_q4& B0 = sh ? a.s0 : a.b0;
    Q4Ptr pp[NP];
    pp[0] = q4_expert(B0, sh ? 0 : e);
    if (GATEUP) pp[NP - 1] = q4_expert(sh ? a.s1 : a.b1, sh ? 0 : e);
    const CUtensorMap* tm[NP];
    tm[0] = sh ? &a.tm_s0 : &a.tm_b0;
    if (GATEUP) tm[NP - 1] = sh ? &a.tm_s1 : &a.tm_b1;
    const int N = B0.out, K = B0.in, G = K >> 5;
    const int nch = (K + 127) >> 7;
    const int row0 = rb * 16 * MT;
    if (row0 >= N) continue;  // warp-uniform
    const int trow = (sh ? 0 : e * N) + row0;   // first row in the bank's 2-D view

    int soff[MT][2];
    bool rv[MT][2];
#pragma unroll
    for (int m = 0; m < MT; ++m)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int row = row0 + 16 * m + g + 8 * h;
        rv[m][h] = row < N;
        soff[m][h] = (rv[m][h] ? row : 0) * G + 2 * (c & 1);
      }
    const int tb = g >> 2, ts = c >> 1;
    const bool xbv = blane && tb < cnt, xsv = ts < cnt;
    int64_t rb_ = 0, rs_ = 0;
    if (xbv) rb_ = a.src_rows ? __ldg(a.src_rows + p0 + tb) : p0 + tb;
    if (!XMMA && xsv) rs_ = a.src_rows ? __ldg(a.src_rows + p0 + ts) : p0 + ts;
    const uint16_t* xb = a.x + rb_ * a.ldx + c * 32;
    const float* xsp = XMMA ? a.xsum : a.xsum + rs_ * a.ldxs + 2 * (c & 1);

    auto issue = [&](int ch) {
      const uint32_t st = ring + st_issue * S::kBytes;
      if (lane == 0) {
        const uint32_t bar = bar0 + 8 * st_issue;
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        mbar_expect(bar, NP * S::kWRows * 64);
#pragma unroll
        for (int p = 0; p < NP; ++p) tma_load_2d(st + p * S::kWRows * 64, tm[p], ch * 16, trow, bar);
      }
      const bool sok = 4 * ch + 2 * (c & 1) < G;
      if (EVEN) {
#pragma unroll
        for (int p = 0; p < NP; ++p)
#pragma unroll
          for (int m = 0; m < MT; ++m) {
            const uint32_t d = st + S::kW + ((p * MT + m) * 32 + lane) * 16;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              cp4(d + 8 * h, pp[p].s + soff[m][h] + ch * 4, rv[m][h] && sok);
              cp4(d + 8 * h + 4, pp[p].b + soff[m][h] + ch * 4, rv[m][h] && sok);
            }
          }
      }
      const int nbytes = (xbv && 4 * ch + c < G) ? 16 : 0;
#pragma unroll
      for (int i = 0; i < 4; ++i)
        cp16_if(st + S::kW + S::kS + (i * 8 + g) * 16, xb + ch * 128 + 8 * i, nbytes, blane);
      if (!XMMA) cp8(st + S::kW + S::kS + S::kX + lane * 8, xsp + ch * 4, xsv && sok);
      st_issue = st_issue == kStages - 1 ? 0 : st_issue + 1;
    };

    float acc[NP][MT][2];
#pragma unroll
    for (int p = 0; p < NP; ++p)
#pragma unroll
      for (int m = 0; m < MT; ++m) acc[p][m][0] = acc[p][m][1] = 0.f;

#pragma unroll
    for (int s = 0; s < kStages - 1; ++s) {
      if (s < nch) issue(s);
      cp_commit();
    }
    for (int ch = 0; ch < nch; ++ch) {
      if (ch + kStages - 1 < nch) issue(ch + kStages - 1);
      cp_commit();
      cp_wait<kStages - 1>();
      const uint32_t st = ring + st_use * S::kBytes;
      if (!mbar_wait(bar0 + 8 * st_use, (parity_bits >> st_use) & 1u)) timed_out = true;
      parity_bits ^= 1u << st_use;

      uint32_t bq[16];
      const uint32_t xa = blane ? st + S::kW + S::kS + g * 16 : zaddr;
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
        const uint2 v = lds64(st + S::kW + S::kS + S::kX + lane * 8);
        xs0 = __uint_as_float(v.x);
        xs1 = __uint_as_float(v.y);
      }
      const int gA = 4 * ch + 2 * (c & 1);   // groups of D columns 2c, 2c+1
#pragma unroll
      for (int p = 0; p < NP; ++p) {
#pragma unroll
        for (int m = 0; m < MT; ++m) {
          const uint32_t wrow = st + p * S::kWRows * 64 + (16 * m + g) * 64 + c * 16;
          const uint4 wg = lds128(wrow), w8 = lds128(wrow + 8 * 64);
          const uint32_t ag[4] = {wg.x, wg.y, wg.z, wg.w};
          const uint32_t a8[4] = {w8.x, w8.y, w8.z, w8.w};
          // One accumulator chain over the chunk's eight MMAs (the resident
          // warps hide its latency; a second chain cost more instructions
          // than it saved).  The tiled kernel uses the same order.
          float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int mm = 0; mm < 8; mm += 2) {
            const int wi = mm >> 1;
            mma16816(d, nib_pair128(ag[wi]), nib_pair128(a8[wi]), nib_pair128(ag[wi] >> 4),
                     nib_pair128(a8[wi] >> 4), bq[2 * mm], bq[2 * mm + 1]);
            mma16816(d, nib_pair128(ag[wi] >> 8), nib_pair128(a8[wi] >> 8),
                     nib_pair128(ag[wi] >> 12), nib_pair128(a8[wi] >> 12), bq[2 * mm + 2],
                     bq[2 * mm + 3]);
          }
          float sc[2][4];   // [h] {s0, s1, b0, b1}
          if (EVEN) {
            const uint4 sb = lds128(st + S::kW + ((p * MT + m) * 32 + lane) * 16);
            const uint32_t sw[4] = {sb.x, sb.y, sb.z, sb.w};
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              sc[h][0] = __uint_as_float(sw[2 * h] << 16);
              sc[h][1] = __uint_as_float(sw[2 * h] & 0xFFFF0000u);
              sc[h][2] = __uint_as_float(sw[2 * h + 1] << 16);
              sc[h][3] = __uint_as_float(sw[2 * h + 1] & 0xFFFF0000u);
            }
          } else {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const bool ok0 = rv[m][h] && gA < G, ok1 = rv[m][h] && gA + 1 < G;
              const int64_t mi = soff[m][h] + ch * 4;
              sc[h][0] = ok0 ? bf16_to_f32(pp[p].s[mi]) : 0.f;
              sc[h][1] = ok1 ? bf16_to_f32(pp[p].s[mi + 1]) : 0.f;
              sc[h][2] = ok0 ? bf16_to_f32(pp[p].b[mi]) : 0.f;
              sc[h][3] = ok1 ? bf16_to_f32(pp[p].b[mi + 1]) : 0.f;
            }
          }
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            // bias - 128*scale: the lop3 operands carry q + 128.
            const float c0 = fmaf(-128.f, sc[h][0], sc[h][2]);
            const float c1 = fmaf(-128.f, sc[h][1], sc[h][3]);
            float v = acc[p][m][h];
            v = fmaf(sc[h][0], d[2 * h], v);
            v = fmaf(c0, xs0, v);
            v = fmaf(sc[h][1], d[2 * h + 1], v);
            v = fmaf(c1, xs1, v);
            acc[p][m][h] = v;
          }
        }
      }
      __syncwarp();   // the stage is read out before the warp refills it
      st_use = st_use == kStages - 1 ? 0 : st_use + 1;
    }

    // lanes c and c^1 hold the two group halves of the same (row, token)
#pragma unroll
    for (int p = 0; p < NP; ++p)
#pragma unroll
      for (int m = 0; m < MT; ++m)
#pragma unroll
        for (int h = 0; h < 2; ++h) acc[p][m][h] += __shfl_xor_sync(0xFFFFFFFFu, acc[p][m][h], 1);
    const int tok = c >> 1;
    if ((c & 1) == 0 && tok < cnt) {
      const int pos = p0 + tok;
      const int64_t dst = a.dst_rows ? __ldg(a.dst_rows + pos) : pos;
#pragma unroll
      for (int m = 0; m < MT; ++m)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          if (!rv[m][h]) continue;
          const int row = row0 + 16 * m + g + 8 * h;
          if (GATEUP) {
            // h is the next projection's input: store it in B order.
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

// ---- host side --------------------------------------------------------------

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// The packed words of a bank as a 2-D tensor [experts*out rows][in/8 words];
// box = 16 words (64 B) x box_rows rows; out-of-range reads fill zeros.
static cudaError_t encode_bank(CUtensorMap* m, const vx_q4& b, int box_rows) {
  auto fn = encode_fn();
  if (!fn) return cudaErrorNotSupported;
  const cuuint64_t dims[2] = {cuuint64_t(b.in / 8), cuuint64_t(b.experts) * cuuint64_t(b.out)};
  const cuuint64_t strides[1] = {cuuint64_t(b.in / 8) * 4};
  const cuuint32_t box[2] = {16, cuuint32_t(box_rows)};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<uint32_t*>(b.w), dims, strides,
                        box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

template <bool GATEUP, int MT, bool XMMA, bool EVEN>
static cudaError_t launch_mma_t(MmaArgs a, int max_items, int max_out, cudaStream_t st) {
  constexpr int NP = GATEUP ? 2 : 1;
  cudaError_t err = encode_bank(&a.tm_b0, a.b0, 16 * MT);
  if (err == cudaSuccess && GATEUP) err = encode_bank(&a.tm_b1, a.b1, 16 * MT);
  if (err == cudaSuccess && a.s0.w) err = encode_bank(&a.tm_s0, a.s0, 16 * MT);
  if (err == cudaSuccess && GATEUP && a.s1.w) err = encode_bank(&a.tm_s1, a.s1, 16 * MT);
  if (err != cudaSuccess) return err;
  a.tiles_per_item = (max_out + 16 * MT - 1) / (16 * MT);
  const size_t smem = size_t(kWarps) * kStages * Stage<NP, MT, XMMA>::kBytes;
  auto kern = gemv_mma_kernel<GATEUP, MT, XMMA, EVEN>;
  err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (err != cudaSuccess) return err;
  const int64_t warps = int64_t(max_items) * a.tiles_per_item;
  const int64_t cap = int64_t(sm_count()) * 2;  // two resident CTAs per SM, persistent
  int64_t grid = (warps + kWarps - 1) / kWarps;
  if (grid > cap) grid = cap;
  if (grid <= 0) return cudaSuccess;
  return launch_streaming(kern, dim3(int(grid)), dim3(kMmaThreads), smem, st, a);
}

template <bool GATEUP, int MT, bool XMMA>
static cudaError_t launch_even(const MmaArgs& a, bool even, int max_items, int max_out, cudaStream_t st) {
  return even ? launch_mma_t<GATEUP, MT, XMMA, true>(a, max_items, max_out, st)
              : launch_mma_t<GATEUP, MT, XMMA, false>(a, max_items, max_out, st);
}

cudaError_t launch_gemv_mma(bool gateup, const MmaArgs& a, int max_items, int max_out,
                            cudaStream_t st) {
  // Even group counts (every input width that is a multiple of 64) copy the
  // scales with the pipeline; odd ones read them directly.
  bool even = (a.b0.in / 32) % 2 == 0;
  if (a.s0.w) even = even && (a.s0.in / 32) % 2 == 0;
  const bool xmma = a.xsum == nullptr;
  if (gateup) {
    return xmma ? launch_even<true, 1, true>(a, even, max_items, max_out, st)
                : launch_even<true, 1, false>(a, even, max_items, max_out, st);
  }
  // gate/up holds two projections per row block: one m-tile each.  The
  // single projection takes 32-row tiles when there is plenty of work.
  const int64_t rows_work = int64_t(max_items) * max_out;
  const bool small = rows_work < int64_t(sm_count()) * 16 * 32;
  if (xmma) return small ? launch_even<false, 1, true>(a, even, max_items, max_out, st)
                         : launch_even<false, 2, true>(a, even, max_items, max_out, st);
  return small ? launch_even<false, 1, false>(a, even, max_items, max_out, st)
               : launch_even<false, 2, false>(a, even, max_items, max_out, st);
}

}  // namespace vx
