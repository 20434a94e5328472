// Persistent grouped Q4 expert GEMM over the tiled pool (sm_100a, tcgen05 +
// TMEM): the prefill-sized sorted gather_qmm of models/flashnext/
// expert_cache.py:2017-2037.
//
// Work: tasks (item, 128-row output tile), an item being an expert's run of
// up to 64 sorted positions; each CTA (one per SM) walks the task list with a
// stride of gridDim.x.  "Swap AB" MMA:
//
//   D[128 weight rows][N tokens] += A[128 rows][K] . B[N tokens][K]^T
//
// A = the dequantised weights (bf16, K-major, 128-byte swizzle) built in
// shared memory from the pool's records; B = the item's activation rows
// (bf16, B order, by TMA with the same swizzle); fp32 accumulators in TMEM,
// double-buffered so one tile's epilogue overlaps the next tile's mainloop.
// Dequantisation follows MLX's affine rule w = bf16(scale*q + bias)
// (metal_runtime.py:1026-1027).
//
// Warp roles (448 threads):
//   warp 0      lane 0: bulk copies of the tile's pool records (weights and
//               scales, 2,560 bytes per 16 or 32 rows) and the TMA copies of
//               B, onto the stage's `full` mbarrier;
//   warp 1      allocates TMEM; lane 0 issues the tcgen05.mma chain, commits
//               each stage back to the producers and each tile to the
//               epilogue;
//   warps 2-9   dequantise: thread = (row, half of the 128-input chunk),
//               records -> registers -> bf16 A tile;
//   warps 10-13 epilogue: TMEM -> registers -> h (SwiGLU) or the outputs.
// Every mbarrier wait is bounded; on expiry bit 9 of the error word is set
// and the kernel carries on, so a broken pipeline reports instead of hanging.
#include "vx_async.cuh"
#include "vx_common.cuh"
#include "vx_launch.h"
#include "vx_tc.cuh"

namespace vx {

constexpr int kPoolThreads = 448;
constexpr int kPoolDequantWarps = 8;

template <bool GATEUP>
struct PoolCfg {
  static constexpr int NP = GATEUP ? 2 : 1;
  static constexpr int kStages = GATEUP ? 2 : 3;
  static constexpr int kBn = kPoolGemmItemChunk;           // token rows of a B tile (max)
  static constexpr int kA = NP * 2 * kAtomBytes;           // A tiles, 128 inputs
  static constexpr int kBAtom = kBn * 128;                 // one 64-input B atom
  static constexpr int kB = 2 * kBAtom;
  static constexpr int kRec = NP * 8 * kTileRecordUnit;    // a 128-row tile's records, 128 inputs
  static constexpr int kStage = kA + kB + kRec;            // every part 1024-byte aligned
  static constexpr int kAccCols = NP * kBn;                // TMEM columns per accumulator buffer
  static constexpr int kTmemCols = 2 * kAccCols;           // two buffers (a power of two)
  static constexpr size_t kSmem = size_t(kStages) * kStage + 1024;
  static_assert(kA % 1024 == 0 && kB % 1024 == 0 && kRec % 1024 == 0, "stage alignment");
};

struct PoolTask {
  int e, p0, cnt, row0, N, K, nch;
  bool sh;
};

VX_DEVICE bool pool_task(const PoolGemmArgs& a, int t, PoolTask& k) {
  const int item = t / a.row_tiles, rt = t - item * a.row_tiles;
  k.e = __ldg(a.items + 3 * item);
  k.p0 = __ldg(a.items + 3 * item + 1);
  k.cnt = __ldg(a.items + 3 * item + 2);
  k.sh = k.e == a.E;
  k.N = k.sh ? a.N_s : a.N_b;
  k.K = k.sh ? a.K_s : a.K_b;
  k.row0 = rt * kGemmRows;
  k.nch = (k.K + 127) >> 7;
  return k.row0 < k.N && k.cnt > 0;
}

template <bool GATEUP>
__global__ void __launch_bounds__(kPoolThreads, 1) gemm_pool_kernel(const __grid_constant__ PoolGemmArgs a) {
  using C = PoolCfg<GATEUP>;
  constexpr int S = C::kStages, NP = C::NP;
  extern __shared__ unsigned char smem_raw[];
  __shared__ __align__(8) uint64_t full[S], a_full[S], empty[S], acc_full[2], tmem_empty[2];
  __shared__ uint32_t tmem_slot;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;
  auto sa = [&](int s, int p) { return base + s * C::kStage + p * 2 * kAtomBytes; };
  auto sb = [&](int s) { return base + s * C::kStage + C::kA; };
  auto sr = [&](int s) { return base + s * C::kStage + C::kA + C::kB; };

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init_n(smem_u32(&full[s]), 1);
      mbar_init_n(smem_u32(&a_full[s]), kPoolDequantWarps);
      mbar_init_n(smem_u32(&empty[s]), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init_n(smem_u32(&acc_full[b]), 1);
      mbar_init_n(smem_u32(&tmem_empty[b]), 4);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) tmem_alloc(smem_u32(&tmem_slot), C::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  const int total = *a.n_items * a.row_tiles;
  const int rec_rows = a.tile_rows, MT = rec_rows >> 4;
  const int rec_bytes = NP * MT * kTileRecordUnit;
  bool timed_out = false;

  if (warp == 0) {
    // ---- producer: records + B tile per chunk
    if (lane == 0) {
      const uint64_t pol_w = policy_evict_first();
      int it = 0;
      for (int t = blockIdx.x; t < total; t += gridDim.x) {
        PoolTask k;
        if (!pool_task(a, t, k)) continue;
        const int bn = k.cnt <= 16 ? 16 : k.cnt <= 32 ? 32 : 64;
        const CUtensorMap* tm = &a.tm[k.sh ? 1 : 0][bn == 16 ? 0 : bn == 32 ? 1 : 2];
        const int rb0 = k.row0 / rec_rows;
        const int rb_total = (k.N + rec_rows - 1) / rec_rows;
        int nrec = kGemmRows / rec_rows;
        if (rb0 + nrec > rb_total) nrec = rb_total - rb0;
        const unsigned char* ebase = k.sh ? a.rec_s : a.rec_b + int64_t(k.e) * a.stride_b;
        const uint32_t bytes = uint32_t(nrec * rec_bytes + 2 * bn * 128);
        for (int ch = 0; ch < k.nch; ++ch, ++it) {
          const int s = it % S;
          const uint32_t ph = uint32_t(it / S) & 1u;
          if (!mbar_wait(smem_u32(&empty[s]), ph ^ 1u)) timed_out = true;
          const uint32_t bar = smem_u32(&full[s]);
          mbar_expect(bar, bytes);
          for (int i = 0; i < nrec; ++i)
            bulk_load(sr(s) + i * rec_bytes, ebase + (int64_t(rb0 + i) * k.nch + ch) * rec_bytes, rec_bytes, bar,
                      pol_w);
          tma_load_2d(sb(s), tm, ch * 128, k.p0, bar);
          tma_load_2d(sb(s) + C::kBAtom, tm, ch * 128 + 64, k.p0, bar);
        }
      }
    }
  } else if (warp == 1) {
    // ---- MMA issue
    if (lane == 0) {
      int it = 0, j = 0;
      for (int t = blockIdx.x; t < total; t += gridDim.x) {
        PoolTask k;
        if (!pool_task(a, t, k)) continue;
        const int buf = j & 1;
        const uint32_t tph = uint32_t(j >> 1) & 1u;
        ++j;
        if (!mbar_wait(smem_u32(&tmem_empty[buf]), tph ^ 1u)) timed_out = true;
        tc_fence_after();
        const uint32_t d0 = tmem + buf * C::kAccCols;
        const uint32_t idesc = mma_idesc((k.cnt + 15) & ~15);
        for (int ch = 0; ch < k.nch; ++ch, ++it) {
          const int s = it % S;
          const uint32_t ph = uint32_t(it / S) & 1u;
          if (!mbar_wait(smem_u32(&a_full[s]), ph)) timed_out = true;
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint32_t koff = (kk & 3) * 32;
            const uint64_t bd = sw128_desc(sb(s) + (kk >> 2) * C::kBAtom + koff);
            const bool acc = ch > 0 || kk > 0;
            mma_bf16(d0, sw128_desc(sa(s, 0) + (kk >> 2) * kAtomBytes + koff), bd, idesc, acc);
            if (GATEUP)
              mma_bf16(d0 + C::kBn, sw128_desc(sa(s, 1) + (kk >> 2) * kAtomBytes + koff), bd, idesc, acc);
          }
          mma_commit(smem_u32(&empty[s]));
        }
        mma_commit(smem_u32(&acc_full[buf]));
      }
    }
  } else if (warp < 2 + kPoolDequantWarps) {
    // ---- dequantise: thread = (row r of the tile, half hf of the chunk)
    const int dt = threadIdx.x - 64;
    const int r = dt & 127, hf = dt >> 7;
    const int ri = r / rec_rows, rl = r - ri * rec_rows;
    const int m = rl >> 4, g = rl & 7, h = (rl >> 3) & 1;
    const uint32_t swz = uint32_t(r & 7);
    int it = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x) {
      PoolTask k;
      if (!pool_task(a, t, k)) continue;
      const bool rv = k.row0 + r < k.N;
      for (int ch = 0; ch < k.nch; ++ch, ++it) {
        const int s = it % S;
        const uint32_t ph = uint32_t(it / S) & 1u;
        if (!mbar_wait(smem_u32(&full[s]), ph)) timed_out = true;
        const uint32_t rec = sr(s) + ri * rec_bytes;
#pragma unroll
        for (int p = 0; p < NP; ++p) {
          const uint32_t rowaddr = sa(s, p) + hf * kAtomBytes + r * 128;
          if (rv) {
            const uint32_t wbase = rec + (p * MT + m) * 1024 + h * 512 + (g * 4 + 2 * hf) * 16;
            const uint4 w0 = lds128(wbase), w1 = lds128(wbase + 16);
            const uint2 sbv = lds64(rec + NP * MT * 1024 + (p * MT + m) * 256 + (g * 2 + hf) * 16 + h * 8);
            const uint32_t s0 = (sbv.x & 0xFFFFu) * 0x10001u, s1 = (sbv.x >> 16) * 0x10001u;
            const uint32_t b0 = (sbv.y & 0xFFFFu) * 0x10001u, b1 = (sbv.y >> 16) * 0x10001u;
            const uint32_t wj[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
            for (int u = 0; u < 8; ++u)
              sts128(rowaddr + ((uint32_t(u) ^ swz) << 4), dequant_word(wj[u], u < 4 ? s0 : s1, u < 4 ? b0 : b1));
          } else {
#pragma unroll
            for (int u = 0; u < 8; ++u) sts128(rowaddr + ((uint32_t(u) ^ swz) << 4), make_uint4(0, 0, 0, 0));
          }
        }
        // generic-proxy writes -> visible to the tensor core's async proxy
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_u32(&a_full[s]));
      }
    }
  } else {
    // ---- epilogue: warps 10..13 cover TMEM lane quarters 2, 3, 0, 1
    const int quarter = warp & 3;
    int j = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x) {
      PoolTask k;
      if (!pool_task(a, t, k)) continue;
      const int buf = j & 1;
      const uint32_t tph = uint32_t(j >> 1) & 1u;
      ++j;
      if (!mbar_wait(smem_u32(&acc_full[buf]), tph)) timed_out = true;
      __syncwarp();   // tcgen05.ld is warp-collective
      tc_fence_after();
      const int erow = k.row0 + quarter * 32 + lane;
      const uint32_t tq = tmem + (uint32_t(quarter * 32) << 16) + buf * C::kAccCols;
      const int nmma = (k.cnt + 15) & ~15;
      for (int cb = 0; cb * 16 < nmma; ++cb) {
        float gv[16], uv[16];
        tmem_ld16(tq + cb * 16, gv);
        if (GATEUP) tmem_ld16(tq + C::kBn + cb * 16, uv);
        if (erow < k.N) {
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int tok = cb * 16 + i;
            if (tok >= k.cnt) break;
            const int64_t pos = k.p0 + tok;
            if (GATEUP) {
              const float hv = silu_mul_bf16(bf16r(gv[i]), bf16r(uv[i]));
              a.out[pos * a.ldo + b_order_col(erow)] = f32_to_bf16(hv);
            } else {
              a.out[pos * a.ldo + erow] = f32_to_bf16(gv[i]);
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&tmem_empty[buf]));
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, C::kTmemCols);
  }
  if (timed_out && a.err) atomicOr(a.err, 0x200);
}

cudaError_t launch_gemm_pool(bool gateup, PoolGemmArgs a, const uint16_t* x, int64_t rows, int64_t ldx,
                             int max_items, cudaStream_t st) {
  if (rows <= 0 || max_items <= 0) return cudaSuccess;
  if (a.tile_rows != 16 && a.tile_rows != 32) return cudaErrorInvalidValue;
  const int Ks = a.rec_s ? a.K_s : a.K_b;
  const int boxes[3] = {16, 32, 64};
  for (int i = 0; i < 3; ++i) {
    cudaError_t e = encode_rows(&a.tm[0][i], x, rows, a.K_b, ldx, boxes[i]);
    if (e == cudaSuccess) e = encode_rows(&a.tm[1][i], x, rows, Ks, ldx, boxes[i]);
    if (e != cudaSuccess) return e;
  }
  const int Nmax = a.rec_s && a.N_s > a.N_b ? a.N_s : a.N_b;
  a.row_tiles = (Nmax + kGemmRows - 1) / kGemmRows;
  const int64_t tasks = int64_t(max_items) * a.row_tiles;
  if (tasks > 0x7FFFFFFF) return cudaErrorInvalidValue;
  a.max_tasks = int(tasks);
  const int grid = int(tasks < sm_count() ? tasks : sm_count());
  if (gateup) {
    auto k = gemm_pool_kernel<true>;
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(PoolCfg<true>::kSmem));
    if (e != cudaSuccess) return e;
    k<<<grid, kPoolThreads, PoolCfg<true>::kSmem, st>>>(a);
  } else {
    auto k = gemm_pool_kernel<false>;
    cudaError_t e =
        cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(PoolCfg<false>::kSmem));
    if (e != cudaSuccess) return e;
    k<<<grid, kPoolThreads, PoolCfg<false>::kSmem, st>>>(a);
  }
  return cudaGetLastError();
}

}  // namespace vx
