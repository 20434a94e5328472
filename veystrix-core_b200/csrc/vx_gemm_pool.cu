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
// A = the dequantised weights (bf16; row m in TMEM lane m, two K values per
// 32-bit column), written into TMEM by the CTA itself from the pool's
// records; B = the item's activation rows (bf16, K-major, B order, by TMA
// with the 128-byte swizzle); fp32 accumulators in TMEM, double-buffered so
// one tile's epilogue overlaps the next tile's mainloop.  Dequantisation
// follows MLX's affine rule w = bf16(scale*q + bias) (metal_runtime.py:
// 1026-1027).  TMEM columns: [accumulator buffers][A ring].
//
// Three rings, each with its own producer, keep the latencies off the tensor
// core's path: records (one 128-input chunk of the tile's pool records per
// stage, from HBM, in shared memory), B (one 64-input atom of activation
// rows per stage, mostly from L2, eight deep, shared memory), and A (the
// dequantised weights of 128 or 64 inputs per stage, in TMEM).  The TMEM
// stores of one A stage take a long round trip (store, wait, fence, arrive),
// so four groups of dequantising warps work on four stages at once.
//
// Warp roles:
//   warp 0       lane 0: bulk copies of the tile's pool records (weights and
//                scales, 2,560 bytes per 16 or 32 rows) into the record ring;
//   warp 1       lane 0: TMA copies of the B rows into the B ring;
//   warp 2       allocates TMEM; lane 0 issues the tcgen05.mma chain, commits
//                each A and B stage back to its producer and each tile to the
//                epilogue;
//   warps 3-18   dequantise: four groups of four warps (one per TMEM lane
//                quarter); thread = one row of A, a whole A stage per group;
//   warps 19-22  epilogue: TMEM -> registers -> h (SwiGLU) or the outputs.
// Every mbarrier wait is bounded; on expiry bit 9 of the error word is set
// and the kernel carries on, so a broken pipeline reports instead of hanging.
#include "vx_async.cuh"
#include "vx_common.cuh"
#include "vx_launch.h"
#include "vx_tc.cuh"

namespace vx {

constexpr int kPoolDequantWarp0 = 3;
constexpr int kPoolGroups = 4;
constexpr int kPoolDequantWarps = 4 * kPoolGroups;
constexpr int kPoolEpiWarp0 = kPoolDequantWarp0 + kPoolDequantWarps;
constexpr int kPoolThreads = 32 * (kPoolEpiWarp0 + 4);

template <bool GATEUP>
struct PoolCfg {
  static constexpr int NP = GATEUP ? 2 : 1;
  static constexpr int kAps = GATEUP ? 1 : 2;              // 64-input atoms per A/B stage
  static constexpr int kStagesPerChunk = 2 / kAps;
  static constexpr int kBn = kPoolGemmItemChunk;           // token rows of a B tile (max)
  static constexpr int kBAtom = kBn * 128;                 // one 64-input B atom
  static constexpr int kBStages = 8;                       // B ring: one 64-input atom per stage
  static constexpr int kRec = NP * 8 * kTileRecordUnit;    // a 128-row tile's records, 128 inputs
  static constexpr int kRecStages = GATEUP ? 6 : 12;
  // TMEM columns per accumulator buffer: two accumulators (gate and up, or
  // the even and odd 64-input atoms of the single projection - a dependent
  // chain of MMAs into one accumulator issues at ~173 cycles per MMA, two
  // interleaved chains at ~130)
  static constexpr int kAccCols = 2 * kBn;
  // TMEM: two accumulator buffers, then the A ring (32 columns = 64 bf16 per
  // projection and atom and lane)
  static constexpr int kACols = NP * kAps * 32;
  static constexpr int kAStages = 4;
  static constexpr int kAcol0 = 2 * kAccCols;
  static constexpr int kTmemCols = 512;
  static_assert(kAcol0 + kAStages * kACols <= kTmemCols, "TMEM columns");
  static constexpr size_t kSmem = size_t(kBStages) * kBAtom + size_t(kRecStages) * kRec + 1024;
  static_assert(kBAtom % 1024 == 0 && kRec % 1024 == 0, "stage alignment");
  static_assert(kSmem <= 227 * 1024, "shared memory");
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
  chain_wait();
  using C = PoolCfg<GATEUP>;
  constexpr int AS = C::kAStages, BS = C::kBStages, RS = C::kRecStages, NP = C::NP, APS = C::kAps;
  extern __shared__ unsigned char smem_raw[];
  __shared__ __align__(8) uint64_t rfull[RS], rempty[RS], afull[AS], aempty[AS], bfull[BS], bempty[BS];
  __shared__ __align__(8) uint64_t acc_full[2], tmem_empty[2];
  __shared__ uint32_t tmem_slot;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;
  // shared memory: the B ring (one atom per stage), then the records ring;
  // the A ring lives in TMEM (acol)
  auto sb = [&](int b) { return base + b * C::kBAtom; };
  auto sr = [&](int r) { return base + BS * C::kBAtom + r * C::kRec; };
  auto acol = [&](int s) { return uint32_t(C::kAcol0 + s * C::kACols); };

  if (threadIdx.x == 0) {
    for (int r = 0; r < RS; ++r) {
      mbar_init_n(smem_u32(&rfull[r]), 1);
      // the four warps of each group owning a stage of the chunk
      mbar_init_n(smem_u32(&rempty[r]), 4 * C::kStagesPerChunk);
    }
    for (int s = 0; s < AS; ++s) {
      mbar_init_n(smem_u32(&afull[s]), 4);
      mbar_init_n(smem_u32(&aempty[s]), 1);
    }
    for (int b = 0; b < BS; ++b) {
      mbar_init_n(smem_u32(&bfull[b]), 1);
      mbar_init_n(smem_u32(&bempty[b]), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init_n(smem_u32(&acc_full[b]), 1);
      mbar_init_n(smem_u32(&tmem_empty[b]), 4);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 2) tmem_alloc(smem_u32(&tmem_slot), C::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  const int total = *a.n_items * a.row_tiles;
  const int rec_rows = a.tile_rows, MT = rec_rows >> 4;
  const int sb_unit = tile_unit_bytes(a.group) - 1024;   // scale/bias bytes per (p, m)
  const int rec_bytes = NP * MT * tile_unit_bytes(a.group);
  bool timed_out = false;

  if (warp == 0) {
    // ---- records producer: one record stage per 128-input chunk, bulk
    // copies by lane 0 onto the stage's mbarrier
    if (lane == 0) {
      const uint64_t pol_w = policy_evict_first();
      int ic = 0;
      for (int t = blockIdx.x; t < total; t += gridDim.x) {
        PoolTask k;
        if (!pool_task(a, t, k)) continue;
        const int rb0 = k.row0 / rec_rows;
        const int rb_total = (k.N + rec_rows - 1) / rec_rows;
        int nrec = kGemmRows / rec_rows;
        if (rb0 + nrec > rb_total) nrec = rb_total - rb0;
        const unsigned char* ebase =
            k.sh ? a.rec_s : a.rec_b + routed_record(a.slot_of, a.slots, k.e) * a.stride_b;
        for (int ch = 0; ch < k.nch; ++ch, ++ic) {
          const int r = ic % RS;
          const uint32_t ph = uint32_t(ic / RS) & 1u;
          if (!mbar_wait_spin(smem_u32(&rempty[r]), ph ^ 1u)) timed_out = true;
          const uint32_t bar = smem_u32(&rfull[r]);
          mbar_expect(bar, uint32_t(nrec * rec_bytes));
          for (int i = 0; i < nrec; ++i)
            bulk_load(sr(r) + i * rec_bytes, ebase + (int64_t(rb0 + i) * k.nch + ch) * rec_bytes, rec_bytes, bar,
                      pol_w);
        }
      }
    }
  } else if (warp == 1) {
    // ---- B producer: the item's activation rows, one 64-input atom per stage
    if (lane == 0) {
      int ib = 0;
      for (int t = blockIdx.x; t < total; t += gridDim.x) {
        PoolTask k;
        if (!pool_task(a, t, k)) continue;
        const int bn = k.cnt <= 16 ? 16 : k.cnt <= 32 ? 32 : 64;
        const CUtensorMap* tm = &a.tm[k.sh ? 1 : 0][bn == 16 ? 0 : bn == 32 ? 1 : 2];
        for (int at = 0; at < 2 * k.nch; ++at, ++ib) {
          const int b = ib % BS;
          const uint32_t ph = uint32_t(ib / BS) & 1u;
          if (!mbar_wait_spin(smem_u32(&bempty[b]), ph ^ 1u)) timed_out = true;
          const uint32_t bar = smem_u32(&bfull[b]);
          mbar_expect(bar, uint32_t(bn * 128));
          tma_load_2d(sb(b), tm, at * 64, k.p0, bar);
        }
      }
    }
  } else if (warp == 2) {
    // ---- MMA issue
    if (lane == 0) {
      int ia = 0, ib = 0, j = 0;
      for (int t = blockIdx.x; t < total; t += gridDim.x) {
        PoolTask k;
        if (!pool_task(a, t, k)) continue;
        const int buf = j & 1;
        const uint32_t tph = uint32_t(j >> 1) & 1u;
        ++j;
        if (!mbar_wait_spin(smem_u32(&tmem_empty[buf]), tph ^ 1u)) timed_out = true;
        tc_fence_after();
        const uint32_t d0 = tmem + buf * C::kAccCols;
        const uint32_t idesc = mma_idesc((k.cnt + 15) & ~15);
        bool acc[2] = {false, false};
        for (int ch = 0; ch < k.nch; ++ch) {
          for (int st = 0; st < C::kStagesPerChunk; ++st, ++ia) {
            const int s = ia % AS;
            const uint32_t ph = uint32_t(ia / AS) & 1u;
            if (!mbar_wait_spin(smem_u32(&afull[s]), ph)) timed_out = true;
            int bs[APS];
#pragma unroll
            for (int at = 0; at < APS; ++at, ++ib) {
              bs[at] = ib % BS;
              if (!mbar_wait_spin(smem_u32(&bfull[bs[at]]), uint32_t(ib / BS) & 1u)) timed_out = true;
            }
            tc_fence_after();
            // the two accumulators alternate MMA by MMA, so neither waits on
            // its own previous MMA
#pragma unroll
            for (int kk = 0; kk < 4; ++kk) {
              const uint32_t koff = kk * 32;
#pragma unroll
              for (int at = 0; at < APS; ++at) {
                const uint64_t bd = sw128_desc(sb(bs[at]) + koff);
                const uint32_t a0 = tmem + acol(s) + at * 32 + kk * 8;
                if (GATEUP) {
                  mma_bf16_ts(d0, a0, bd, idesc, acc[0]);
                  mma_bf16_ts(d0 + C::kBn, a0 + 32, bd, idesc, acc[0]);
                  acc[0] = true;
                } else {
                  mma_bf16_ts(d0 + at * C::kBn, a0, bd, idesc, acc[at]);
                  acc[at] = true;
                }
              }
            }
#pragma unroll
            for (int at = 0; at < APS; ++at) mma_commit(smem_u32(&bempty[bs[at]]));
            mma_commit(smem_u32(&aempty[s]));
          }
        }
        mma_commit(smem_u32(&acc_full[buf]));
      }
    }
  } else if (warp < kPoolDequantWarp0 + kPoolDequantWarps) {
    // ---- dequantise.  A warp may only touch its TMEM lane quarter
    // (warp % 4), so a thread owns row 32*quarter + lane of A.  The 16 warps
    // form kPoolGroups groups of four (one per quarter); group g builds the A
    // stages whose running index is g mod kPoolGroups, all of the stage's
    // halves (gate and up, or both atoms), so several stages are in flight
    // while each group waits for its TMEM stores to land.
    const int quarter = warp & 3, grp = (warp - kPoolDequantWarp0) >> 2;
    const int r = quarter * 32 + lane;
    const int ri = r / rec_rows, rl = r - ri * rec_rows;
    const int m = rl >> 4, g = rl & 7, h = (rl >> 3) & 1;
    const uint32_t tq = tmem + (uint32_t(quarter * 32) << 16);
    const uint32_t rrow = ri * rec_bytes + m * 1024 + h * 512 + g * 64;                 // words, p = 0
    // scales, p = 0: groups of 32 {s_a s_b | b_a b_b} per (g, atom) pair of
    // rows; native G64 one {s | b} word per row and 64 inputs ([g][atom][h])
    const bool g64 = a.group == 64;
    const uint32_t srow = ri * rec_bytes + NP * MT * 1024 + m * sb_unit + (g64 ? g * 16 + h * 4 : g * 32 + h * 8);
    int ic = 0, ia = 0;
    for (int t = blockIdx.x; t < total; t += gridDim.x) {
      PoolTask k;
      if (!pool_task(a, t, k)) continue;
      const bool rv = k.row0 + r < k.N;
      for (int ch = 0; ch < k.nch; ++ch, ++ic) {
        const int rs = ic % RS;
        bool mine = false;   // does this group own a stage of this chunk?
        for (int st = 0; st < C::kStagesPerChunk; ++st) mine |= (ia + st) % kPoolGroups == grp;
        if (!mine) {
          ia += C::kStagesPerChunk;
          continue;
        }
        if (!mbar_wait(smem_u32(&rfull[rs]), uint32_t(ic / RS) & 1u)) timed_out = true;
        const uint32_t rec = sr(rs);
        for (int st = 0; st < C::kStagesPerChunk; ++st, ++ia) {
          if (ia % kPoolGroups != grp) continue;
          const int s = ia % AS;
          const uint32_t ph = uint32_t(ia / AS) & 1u;
          // two halves of 64 inputs: (gate, up) of atom st, or atoms 0 and 1;
          // the second half is computed while the first one's store drains
          uint32_t av[32];
#pragma unroll
          for (int hv = 0; hv < 2; ++hv) {
            const int p = GATEUP ? hv : 0, atom = GATEUP ? st : hv;
            uint4 w0 = make_uint4(0, 0, 0, 0), w1 = w0;
            uint2 sbv = make_uint2(0, 0);
            if (rv) {
              const uint32_t wb = rec + rrow + p * MT * 1024 + atom * 32;
              w0 = lds128(wb);
              w1 = lds128(wb + 16);
              if (g64) {
                const uint32_t wsb = lds32(rec + srow + p * MT * sb_unit + atom * 8);
                sbv = make_uint2((wsb & 0xFFFFu) | (wsb << 16), (wsb >> 16) | (wsb & 0xFFFF0000u));
              } else {
                sbv = lds64(rec + srow + p * MT * sb_unit + atom * 16);
              }
            }
            const uint32_t s0 = (sbv.x & 0xFFFFu) * 0x10001u, s1 = (sbv.x >> 16) * 0x10001u;
            const uint32_t b0 = (sbv.y & 0xFFFFu) * 0x10001u, b1 = (sbv.y >> 16) * 0x10001u;
            const uint32_t wj[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
            for (int u = 0; u < 8; ++u) {
              const uint4 o = dequant_word(wj[u], u < 4 ? s0 : s1, u < 4 ? b0 : b1);
              av[4 * u + 0] = rv ? o.x : 0u;
              av[4 * u + 1] = rv ? o.y : 0u;
              av[4 * u + 2] = rv ? o.z : 0u;
              av[4 * u + 3] = rv ? o.w : 0u;
            }
            if (hv == 0) {
              if (!mbar_wait(smem_u32(&aempty[s]), ph ^ 1u)) timed_out = true;
              __syncwarp();   // tcgen05.st is warp-collective
              tc_fence_after();
            }
            tmem_st32(tq + acol(s) + hv * 32, av);   // registers are read at issue
          }
          tmem_wait_st();
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(smem_u32(&afull[s]));
        }
        __syncwarp();   // the warp has read the record stage
        if (lane == 0) mbar_arrive(smem_u32(&rempty[rs]));
      }
    }
  } else {
    // ---- epilogue: the last four warps cover the four TMEM lane quarters
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
        tmem_ld16(tq + C::kBn + cb * 16, uv);   // up, or the odd-atom partial sums
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
              a.out[pos * a.ldo + erow] = f32_to_bf16(gv[i] + uv[i]);
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
  if (warp == 2) {
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
    return launch_streaming(k, dim3(grid), dim3(kPoolThreads), PoolCfg<true>::kSmem, st, a);
  }
  auto k = gemm_pool_kernel<false>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(PoolCfg<false>::kSmem));
  if (e != cudaSuccess) return e;
  return launch_streaming(k, dim3(grid), dim3(kPoolThreads), PoolCfg<false>::kSmem, st, a);
}

}  // namespace vx
