// Grouped Q4 expert GEMM on the 5th-generation tensor cores (sm_100a,
// tcgen05 + TMEM) for prefill-sized batches: the sorted-path gather_qmm of
// models/flashnext/expert_cache.py:2017-2037 when experts see tens of tokens.
//
// One CTA = one work item (an expert's run of up to 128 sorted positions)
// x one 128-row tile of the projection's outputs.  The MMA is "swap AB":
//
//   D[128 weight rows][N tokens] += A[128 rows][K] . B[N tokens][K]^T
//
// with A = the dequantised weights (bf16, K-major, 128-byte swizzle, written
// by the CTA itself) and B = the item's activation rows (bf16, K-major,
// brought by TMA with the same swizzle), fp32 accumulators in TMEM.  The
// dequantisation follows MLX's affine rule w = bf16(scale*q + bias) (one
// rounding of the exact value; metal_runtime.py:1026-1027): one lop3 turns a
// nibble pair into the exact bf16 pair 128+q, one bf16x2 FMA subtracts 128
// exactly, a second applies scale and bias.  Both operands keep the inputs
// of each 8-block in "B order" (x0 x4 x1 x5 x2 x6 x3 x7), the order the
// lop3 produces, so the dot products are those of the natural order.
//
// Warp roles (320 threads):
//   warps 0-7  dequantise the A tile of each 128-input chunk (thread = row,
//              64 inputs), then run the epilogue from TMEM;
//   warp 8     lane 0 issues the TMA copies of the B tile;
//   warp 9     allocates TMEM; lane 0 issues the tcgen05.mma chain and
//              commits each stage back to the producers.
// Gate/up mode keeps two accumulators (gate, up) over the same B and writes
// h = silu(gate)*up with MLX's bf16 sequence; projection mode writes the
// bf16 outputs.  Every mbarrier wait is bounded: on expiry the kernel sets
// bit 9 of the error word and carries on, so a fault in the pipeline is
// reported instead of hanging the GPU.
#include <cudaTypedefs.h>

#include "vx_async.cuh"
#include "vx_common.cuh"
#include "vx_launch.h"
#include "vx_tc.cuh"

namespace vx {

constexpr int kGemmThreads = 320;

template <bool GATEUP>
struct GemmCfg {
  static constexpr int kStages = GATEUP ? 2 : 3;
  static constexpr int kA = 2 * kAtomBytes;                // 128 inputs: two atoms
  static constexpr int kB = 2 * kAtomBytes;                // up to 128 tokens
  static constexpr int kStage = (GATEUP ? 2 : 1) * kA + kB;
  static constexpr int kTmemCols = GATEUP ? 256 : 128;
  static constexpr size_t kSmem = size_t(kStages) * kStage + 1024;   // + alignment slack
};

template <bool GATEUP>
__global__ void __launch_bounds__(kGemmThreads, 1) gemm_tc_kernel(const __grid_constant__ GemmArgs a) {
  chain_wait();
  using C = GemmCfg<GATEUP>;
  constexpr int S = C::kStages;
  extern __shared__ unsigned char smem_raw[];
  __shared__ __align__(8) uint64_t a_full[S], b_full[S], empty[S], acc_full;
  __shared__ uint32_t tmem_slot;

  const int n_items = *a.n_items;
  const int item = blockIdx.x / a.row_tiles, rt = blockIdx.x - item * a.row_tiles;
  if (item >= n_items) return;
  const int e = __ldg(a.items + 3 * item), p0 = __ldg(a.items + 3 * item + 1);
  const int cnt = __ldg(a.items + 3 * item + 2);
  const bool sh = e == a.E;
  const vx_q4& B0 = sh ? a.s0 : a.b0;
  const vx_q4& B1 = sh ? a.s1 : a.b1;
  const int N = B0.out, K = B0.in;
  const int row0 = rt * kGemmRows;
  if (row0 >= N || cnt <= 0) return;   // uniform over the CTA
  const int nch = (K + 127) >> 7;
  const int bn = cnt <= 16 ? 16 : cnt <= 32 ? 32 : cnt <= 64 ? 64 : 128;
  const int nmma = (cnt + 15) & ~15;
  const CUtensorMap* tm = &a.tm[sh ? 1 : 0][bn == 16 ? 0 : bn == 32 ? 1 : bn == 64 ? 2 : 3];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;
  auto stage_a = [&](int s, int p) { return base + s * C::kStage + p * C::kA; };
  auto stage_b = [&](int s) { return base + s * C::kStage + (GATEUP ? 2 : 1) * C::kA; };

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init_n(smem_u32(&a_full[s]), 8);
      mbar_init_n(smem_u32(&b_full[s]), 1);
      mbar_init_n(smem_u32(&empty[s]), 1);
    }
    mbar_init_n(smem_u32(&acc_full), 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 9) {
    tmem_alloc(smem_u32(&tmem_slot), C::kTmemCols);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  bool timed_out = false;

  if (warp < 8) {
    // ---- dequantise A: thread = weight row, 64 inputs (one atom) per chunk
    const int r = threadIdx.x & 127, hf = threadIdx.x >> 7;
    const int grow = row0 + r;
    const bool rv = grow < N;
    const int G = K >> 5, Wn = K >> 3;
    const Q4Ptr q0 = q4_expert(B0, sh ? 0 : e);
    Q4Ptr q1 = q0;
    if (GATEUP) q1 = q4_expert(B1, sh ? 0 : e);
    const uint32_t swz = uint32_t(r & 7);
    for (int ch = 0; ch < nch; ++ch) {
      const int s = ch % S;
      const uint32_t ph = uint32_t(ch / S) & 1u;
      const int k0 = ch * 128 + hf * 64;   // first input of this thread's atom
      uint4 wv[GATEUP ? 2 : 1][2];
      uint32_t sc[GATEUP ? 2 : 1][2], bi[GATEUP ? 2 : 1][2];
#pragma unroll
      for (int p = 0; p < (GATEUP ? 2 : 1); ++p) {
        const Q4Ptr& q = p ? q1 : q0;
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const int kk = k0 + 32 * j;            // one quant group per uint4
          const bool ok = rv && kk < K;
          wv[p][j] = ok ? ldg_nc(q.w + int64_t(grow) * Wn + (kk >> 3)) : make_uint4(0, 0, 0, 0);
          const int64_t gi = int64_t(grow) * G + (kk >> 5);
          const uint32_t sv = ok ? uint32_t(__ldg(q.s + gi)) : 0u;
          const uint32_t bv = ok ? uint32_t(__ldg(q.b + gi)) : 0u;
          sc[p][j] = sv | (sv << 16);
          bi[p][j] = bv | (bv << 16);
        }
      }
      if (!mbar_wait(smem_u32(&empty[s]), ph ^ 1u)) timed_out = true;
#pragma unroll
      for (int p = 0; p < (GATEUP ? 2 : 1); ++p) {
        const uint32_t rowaddr = stage_a(s, p) + hf * kAtomBytes + r * 128;
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const uint32_t wj[4] = {wv[p][j].x, wv[p][j].y, wv[p][j].z, wv[p][j].w};
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const uint4 o = dequant_word(wj[u], sc[p][j], bi[p][j]);
            const uint32_t unit = uint32_t(4 * j + u) ^ swz;
            asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(rowaddr + (unit << 4)), "r"(o.x),
                         "r"(o.y), "r"(o.z), "r"(o.w)
                         : "memory");
          }
        }
      }
      // generic-proxy writes -> visible to the tensor core's async proxy
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&a_full[s]));
    }

    // ---- epilogue: TMEM -> registers -> global
    if (!mbar_wait(smem_u32(&acc_full), 0)) timed_out = true;
    __syncwarp();   // tcgen05.ld is warp-collective
    tc_fence_after();
    const int quarter = warp & 3;
    const int erow = row0 + quarter * 32 + lane;
    const uint32_t tq = tmem + (uint32_t(quarter * 32) << 16);
    for (int cb = warp >> 2; cb * 16 < nmma; cb += 2) {
      float g[16], u[16];
      tmem_ld16(tq + cb * 16, g);
      if (GATEUP) tmem_ld16(tq + 128 + cb * 16, u);
      if (erow < N) {
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int tok = cb * 16 + i;
          if (tok >= cnt) break;
          const int64_t pos = p0 + tok;
          if (GATEUP) {
            const float h = silu_mul_bf16(bf16r(g[i]), bf16r(u[i]));
            a.out[pos * a.ldo + b_order_col(erow)] = f32_to_bf16(h);
          } else {
            a.out[pos * a.ldo + erow] = f32_to_bf16(g[i]);
          }
        }
      }
    }
  } else if (warp == 8) {
    // ---- B tiles by TMA (lane 0)
    if (lane == 0) {
      for (int ch = 0; ch < nch; ++ch) {
        const int s = ch % S;
        const uint32_t ph = uint32_t(ch / S) & 1u;
        if (!mbar_wait(smem_u32(&empty[s]), ph ^ 1u)) timed_out = true;
        const uint32_t bar = smem_u32(&b_full[s]);
        mbar_expect(bar, uint32_t(2 * bn * 128));
        tma_load_2d(stage_b(s), tm, ch * 128, p0, bar);
        tma_load_2d(stage_b(s) + kAtomBytes, tm, ch * 128 + 64, p0, bar);
      }
    }
  } else {
    // ---- MMA issue (warp 9, lane 0)
    if (lane == 0) {
      const uint32_t idesc = mma_idesc(nmma);
      for (int ch = 0; ch < nch; ++ch) {
        const int s = ch % S;
        const uint32_t ph = uint32_t(ch / S) & 1u;
        if (!mbar_wait(smem_u32(&a_full[s]), ph)) timed_out = true;
        if (!mbar_wait(smem_u32(&b_full[s]), ph)) timed_out = true;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t off = (kk >> 2) * kAtomBytes + (kk & 3) * 32;
          const uint64_t bd = sw128_desc(stage_b(s) + off);
          const bool acc = ch > 0 || kk > 0;
          mma_bf16(tmem, sw128_desc(stage_a(s, 0) + off), bd, idesc, acc);
          if (GATEUP) mma_bf16(tmem + 128, sw128_desc(stage_a(s, 1) + off), bd, idesc, acc);
        }
        mma_commit(smem_u32(&empty[s]));
      }
      mma_commit(smem_u32(&acc_full));
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }
  if (timed_out && a.err) atomicOr(a.err, 0x200);
}

// ---- host side --------------------------------------------------------------

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn_gemm() {
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

// bf16 rows [rows][ld] seen as a [rows][K] tensor (columns >= K read as
// zero); box = 64 columns (128 bytes, swizzled) x box_rows rows.
cudaError_t encode_rows(CUtensorMap* m, const uint16_t* p, int64_t rows, int K, int64_t ld,
                               int box_rows) {
  auto fn = encode_fn_gemm();
  if (!fn) return cudaErrorNotSupported;
  const cuuint64_t dims[2] = {cuuint64_t(K), cuuint64_t(rows)};
  const cuuint64_t strides[1] = {cuuint64_t(ld) * 2};
  const cuuint32_t box[2] = {64, cuuint32_t(box_rows)};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<uint16_t*>(p), dims, strides, box,
                        estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

cudaError_t launch_gemm_tc(bool gateup, GemmArgs a, const uint16_t* x, int64_t rows, int64_t ldx,
                           int max_items, cudaStream_t st) {
  if (rows <= 0 || max_items <= 0) return cudaSuccess;
  const int Kb = a.b0.in, Ks = a.s0.w ? a.s0.in : a.b0.in;
  const int boxes[4] = {16, 32, 64, 128};
  for (int i = 0; i < 4; ++i) {
    cudaError_t e = encode_rows(&a.tm[0][i], x, rows, Kb, ldx, boxes[i]);
    if (e == cudaSuccess) e = encode_rows(&a.tm[1][i], x, rows, Ks, ldx, boxes[i]);
    if (e != cudaSuccess) return e;
  }
  const int Nmax = a.s0.w ? (a.b0.out > a.s0.out ? a.b0.out : a.s0.out) : a.b0.out;
  a.row_tiles = (Nmax + kGemmRows - 1) / kGemmRows;
  const int64_t grid = int64_t(max_items) * a.row_tiles;
  if (grid > 0x7FFFFFFF) return cudaErrorInvalidValue;
  if (gateup) {
    auto k = gemm_tc_kernel<true>;
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(GemmCfg<true>::kSmem));
    if (e != cudaSuccess) return e;
    return launch_streaming(k, dim3(int(grid)), dim3(kGemmThreads), GemmCfg<true>::kSmem, st, a);
  }
  auto k = gemm_tc_kernel<false>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(GemmCfg<false>::kSmem));
  if (e != cudaSuccess) return e;
  return launch_streaming(k, dim3(int(grid)), dim3(kGemmThreads), GemmCfg<false>::kSmem, st, a);
}

// x rows (token src_rows[p] for positions p < *n_rows) -> bf16 rows in B
// order, [rows][K]: the B operand of the gate/up GEMM.
__global__ void gather_border_kernel(const uint16_t* __restrict__ x, int64_t ldx, int K,
                                     const int32_t* __restrict__ src_rows, const int32_t* __restrict__ n_rows,
                                     int64_t rows, uint16_t* __restrict__ out) {
  chain_begin();
  const int nb = K / 8;
  const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= rows * nb) return;
  const int64_t p = i / nb;
  if (n_rows && p >= *n_rows) return;
  const int blk = int(i - p * nb);
  const int64_t r = src_rows ? int64_t(__ldg(src_rows + p)) : p;
  const uint4 v = *reinterpret_cast<const uint4*>(x + r * ldx + blk * 8);
  uint4 o;
  o.x = prmt(v.x, v.z, 0x5410);
  o.y = prmt(v.x, v.z, 0x7632);
  o.z = prmt(v.y, v.w, 0x5410);
  o.w = prmt(v.y, v.w, 0x7632);
  *reinterpret_cast<uint4*>(out + p * K + blk * 8) = o;
}

cudaError_t launch_gather_border(const uint16_t* x, int64_t ldx, int K, const int32_t* src_rows,
                                 const int32_t* n_rows, int64_t rows, uint16_t* out, cudaStream_t st) {
  const int64_t n = rows * (K / 8);
  if (n == 0) return cudaSuccess;
  return launch_chained(gather_border_kernel, dim3(int((n + 255) / 256)), dim3(256), 0, st, x, ldx, K,
                        src_rows, n_rows, rows, out);
}

}  // namespace vx
