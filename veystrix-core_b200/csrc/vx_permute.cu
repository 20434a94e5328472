// Stable sort of (token, slot) items by expert id: the permutation of mlx-vlm
// _gather_sort/_scatter_unsort (called at models/flashnext/expert_cache.py:
// 2017-2037), which is a stable argsort of the flat expert ids.
//
// One CTA: a counting pass (shared-memory histogram), an exclusive scan into
// run offsets, then a stable scatter in chunks of blockDim items.  Inside a
// chunk, __match_any_sync groups lanes by expert; the rank of an item is its
// rank among equal lanes of its warp, plus the items of lower warps in the
// chunk with the same expert, plus the items of earlier chunks.  The result
// depends only on the ids, never on scheduling.
#include "vx_common.cuh"
#include "vx_launch.h"

namespace vx {

constexpr int kPermThreads = 1024;
constexpr int kPermWarps = kPermThreads / 32;

__device__ int block_exclusive_scan(int v, int* warp_tot) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int inc = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int n = __shfl_up_sync(0xFFFFFFFFu, inc, o);
    if (lane >= o) inc += n;
  }
  if (lane == 31) warp_tot[warp] = inc;
  __syncthreads();
  if (warp == 0) {
    int t = lane < kPermWarps ? warp_tot[lane] : 0;
    int ti = t;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int n = __shfl_up_sync(0xFFFFFFFFu, ti, o);
      if (lane >= o) ti += n;
    }
    if (lane < kPermWarps) warp_tot[lane] = ti - t;  // exclusive warp base
  }
  __syncthreads();
  const int r = warp_tot[warp] + inc - v;
  __syncthreads();
  return r;
}

// ids [P]; expert E (if shared_items > 0) is appended with shared_items items
// whose x rows are 0..shared_items-1.  shared_items < 0 means offsets has
// only E+1 entries.
__global__ void __launch_bounds__(kPermThreads) permute_kernel(
    const int32_t* __restrict__ ids, int P, int E, int shared_items, int k_div,
    const int32_t* __restrict__ src_map, int32_t* __restrict__ order,
    int32_t* __restrict__ inverse, int32_t* __restrict__ offsets, int32_t* __restrict__ active,
    int32_t* __restrict__ n_active, int32_t* __restrict__ src_rows, int32_t* __restrict__ err,
    int item_chunk, int32_t* __restrict__ items, int32_t* __restrict__ n_items) {
  extern __shared__ int smem[];
  int* counts = smem;                         // [E]
  int* base = counts + E;                     // [E]  run start
  int* running = base + E;                    // [E]  items placed so far
  int* hist = running + E;                    // [kPermWarps][E]
  __shared__ int warp_tot[32];
  __shared__ int s_bad;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

  for (int e = tid; e < E; e += kPermThreads) counts[e] = running[e] = 0;
  for (int i = tid; i < kPermWarps * E; i += kPermThreads) hist[i] = 0;
  if (tid == 0) s_bad = 0;
  __syncthreads();
  for (int i = tid; i < P; i += kPermThreads) {
    const int id = ids[i];
    if (id >= 0 && id < E) atomicAdd(&counts[id], 1);
    else atomicAdd(&s_bad, 1);
  }
  __syncthreads();

  // Exclusive scan of counts and of the "has items" flags, E <= 4 per thread.
  int carry = 0, acarry = 0;
  for (int e0 = 0; e0 < E; e0 += kPermThreads) {
    const int e = e0 + tid;
    const int c = e < E ? counts[e] : 0;
    const int ex = block_exclusive_scan(c, warp_tot);
    const int f = c > 0 ? 1 : 0;
    const int ax = block_exclusive_scan(f, warp_tot);
    if (e < E) {
      base[e] = carry + ex;
      offsets[e] = carry + ex;
      if (f) active[acarry + ax] = e;
    }
    // totals of this slice
    __shared__ int tot_c, tot_a;
    if (tid == kPermThreads - 1) { tot_c = ex + c; tot_a = ax + f; }
    __syncthreads();
    carry += tot_c;
    acarry += tot_a;
    __syncthreads();
  }
  if (tid == 0) {
    offsets[E] = carry;
    // shared_items < 0: the caller's offsets has E+1 entries (no shared run)
    if (shared_items >= 0) offsets[E + 1] = carry + shared_items;
    int na = acarry;
    if (shared_items > 0) active[na++] = E;
    *n_active = na;
    if (err && s_bad) atomicAdd(err, s_bad);
  }
  for (int t = tid; t < shared_items; t += kPermThreads) {
    if (src_rows) src_rows[carry + t] = t;
  }

  // Work items for the grouped kernels: each expert's run cut into chunks of
  // at most item_chunk positions, in expert order: {expert, first, count}.
  if (items) {
    const int na = acarry + (shared_items > 0 ? 1 : 0);
    int icarry = 0;
    for (int a0 = 0; a0 < na; a0 += kPermThreads) {
      const int ai = a0 + tid;
      int e = -1, n = 0, first = 0;
      if (ai < na) {
        e = ai < acarry ? active[ai] : E;
        n = e < E ? counts[e] : shared_items;
        first = e < E ? base[e] : carry;
      }
      const int nch = (n + item_chunk - 1) / item_chunk;
      const int ex = block_exclusive_scan(nch, warp_tot);
      for (int j = 0; j < nch; ++j) {
        int32_t* it = items + 3 * (icarry + ex + j);
        it[0] = e;
        it[1] = first + j * item_chunk;
        it[2] = min(item_chunk, n - j * item_chunk);
      }
      __shared__ int tot_i;
      if (tid == kPermThreads - 1) tot_i = ex + nch;
      __syncthreads();
      icarry += tot_i;
      __syncthreads();
    }
    if (tid == 0) *n_items = icarry;
  }

  // Stable scatter.
  for (int c0 = 0; c0 < P; c0 += kPermThreads) {
    const int i = c0 + tid;
    int key = -1;
    if (i < P) {
      key = ids[i];
      if (key < 0 || key >= E) {
        key = -1;
        inverse[i] = -1;
      }
    }
    const unsigned peers = __match_any_sync(0xFFFFFFFFu, key);
    const int rank = __popc(peers & ((1u << lane) - 1u));
    const bool leader = (__ffs(peers) - 1) == lane;
    if (key >= 0 && leader) hist[warp * E + key] = __popc(peers);
    __syncthreads();
    if (key >= 0) {
      int before = running[key];
      for (int w = 0; w < warp; ++w) before += hist[w * E + key];
      const int pos = base[key] + before + rank;
      order[pos] = i;
      inverse[i] = pos;
      if (src_rows) src_rows[pos] = src_map ? src_map[i] : i / k_div;
    }
    __syncthreads();
    if (key >= 0 && leader) {
      atomicAdd(&running[key], __popc(peers));
      hist[warp * E + key] = 0;
    }
    __syncthreads();
  }
}

cudaError_t launch_permute(const int32_t* ids, int64_t P, int E, int shared_items, int k_div,
                           const int32_t* src_map, int32_t* order, int32_t* inverse,
                           int32_t* offsets, int32_t* active, int32_t* n_active,
                           int32_t* src_rows, int32_t* err, int item_chunk, int32_t* items,
                           int32_t* n_items, cudaStream_t st) {
  const size_t smem = size_t(E) * (3 + kPermWarps) * sizeof(int);
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(permute_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         int(smem));
    if (e != cudaSuccess) return e;
  }
  permute_kernel<<<1, kPermThreads, smem, st>>>(ids, int(P), E, shared_items, k_div, src_map, order,
                                                inverse, offsets, active, n_active, src_rows, err,
                                                item_chunk, items, n_items);
  return cudaGetLastError();
}

// Items of a gather_qmm call: item i = b*M + m has key rhs[b] and x row
// (lhs ? lhs[b] : b)*M + m.  An lhs entry outside the x batch gets key -1,
// so the permutation drops (and counts) the item instead of reading past x.
__global__ void gather_items_kernel(const int32_t* lhs, const int32_t* rhs, int64_t B, int M,
                                    int64_t x_rows, int32_t* keys, int32_t* src_map) {
  const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= B * M) return;
  const int64_t b = i / M, m = i - b * M;
  const int64_t l = lhs ? int64_t(lhs[b]) : b;
  const bool ok = l >= 0 && (l + 1) * M <= x_rows;
  keys[i] = ok ? rhs[b] : -1;
  src_map[i] = ok ? int32_t(l * M + m) : 0;
}

cudaError_t launch_gather_items(const int32_t* lhs, const int32_t* rhs, int64_t B, int M,
                                int64_t x_rows, int32_t* keys, int32_t* src_map, cudaStream_t st) {
  const int64_t n = B * M;
  if (n == 0) return cudaSuccess;
  gather_items_kernel<<<int((n + 255) / 256), 256, 0, st>>>(lhs, rhs, B, M, x_rows, keys, src_map);
  return cudaGetLastError();
}

}  // namespace vx
