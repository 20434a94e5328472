// Stable sort of (token, slot) items by expert id: the permutation of mlx-vlm
// _gather_sort/_scatter_unsort (called at models/flashnext/expert_cache.py:
// 2017-2037), which is a stable argsort of the flat expert ids.
//
// Three phases: a counting pass (shared-memory histogram), an exclusive scan
// into run offsets (plus the active-expert list and the work-item table of
// the grouped kernels), then a stable scatter in chunks of blockDim items.
// Inside a chunk, __match_any_sync groups lanes by expert; the rank of an item
// is its rank among equal lanes of its warp, plus the items of lower warps in
// the chunk with the same expert, plus the items placed before the chunk.
// The result depends only on the ids, never on scheduling.
//
// Decode-sized inputs run all three phases in one CTA.  Prefill-sized inputs
// (more than kPermMultiMin ids) split the ids into slices (perm_slice): one
// CTA per slice counts, one CTA scans the per-slice counts into per-slice
// starting positions (slice order = flat order, so the sort stays stable),
// and one CTA per slice scatters.
#include "vx_common.cuh"
#include "vx_launch.h"
#include "vx_perm_small.cuh"

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

// Histogram of ids[lo, hi) into counts[E] (shared, zeroed by the caller);
// returns the number of ids outside [0, E) (block-wide, valid on all threads
// after the call).
__device__ int perm_count(const int32_t* ids, int64_t lo, int64_t hi, int E, int* counts, int* s_bad) {
  for (int64_t i = lo + threadIdx.x; i < hi; i += kPermThreads) {
    const int id = ids[i];
    if (id >= 0 && id < E) atomicAdd(&counts[id], 1);
    else atomicAdd(s_bad, 1);
  }
  __syncthreads();
  return *s_bad;
}

// From counts[E] (shared): base[e] = offsets[e] (run starts), the active
// list, offsets[E] (and offsets[E+1] with the shared run), the shared run's
// src_rows, and the work-item table.  Returns the number of routed items.
__device__ int perm_offsets(int E, int shared_items, const int* counts, int* base, int* warp_tot,
                            int32_t* offsets, int32_t* active, int32_t* n_active, int32_t* src_rows,
                            int item_chunk, int32_t* items, int32_t* n_items) {
  const int tid = threadIdx.x;
  __shared__ int tot_c, tot_a, tot_i;
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
    if (tid == kPermThreads - 1) {
      tot_c = ex + c;
      tot_a = ax + f;
    }
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
  }
  for (int t = tid; t < shared_items; t += kPermThreads)
    if (src_rows) src_rows[carry + t] = t;

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
      if (tid == kPermThreads - 1) tot_i = ex + nch;
      __syncthreads();
      icarry += tot_i;
      __syncthreads();
    }
    if (tid == 0) *n_items = icarry;
  }
  return carry;
}

// Stable scatter of ids[lo, hi): running[e] (shared) holds the next position
// of expert e; hist is [kPermWarps][E] shared scratch, zeroed.
__device__ void perm_scatter(const int32_t* ids, int64_t lo, int64_t hi, int E, int k_div,
                             const int32_t* src_map, int* running, int* hist, int32_t* order,
                             int32_t* inverse, int32_t* src_rows) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int64_t c0 = lo; c0 < hi; c0 += kPermThreads) {
    const int64_t i = c0 + tid;
    int key = -1;
    if (i < hi) {
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
      const int pos = before + rank;
      order[pos] = int32_t(i);
      inverse[i] = pos;
      if (src_rows) src_rows[pos] = src_map ? src_map[i] : int32_t(i / k_div);
    }
    __syncthreads();
    if (key >= 0 && leader) {
      atomicAdd(&running[key], __popc(peers));
      hist[warp * E + key] = 0;
    }
    __syncthreads();
  }
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
  chain_begin();
  extern __shared__ int smem[];
  int* counts = smem;                         // [E]
  int* base = counts + E;                     // [E]  run start
  int* hist = base + E;                       // [kPermWarps][E]
  __shared__ int warp_tot[32];
  __shared__ int s_bad;
  const int tid = threadIdx.x;
  for (int e = tid; e < E; e += kPermThreads) counts[e] = 0;
  for (int i = tid; i < kPermWarps * E; i += kPermThreads) hist[i] = 0;
  if (tid == 0) s_bad = 0;
  __syncthreads();
  const int bad = perm_count(ids, 0, P, E, counts, &s_bad);
  if (tid == 0 && err && bad) atomicAdd(err, bad);
  perm_offsets(E, shared_items, counts, base, warp_tot, offsets, active, n_active, src_rows, item_chunk,
               items, n_items);
  __syncthreads();
  perm_scatter(ids, 0, P, E, k_div, src_map, base, hist, order, inverse, src_rows);
}

// ---- decode-sized inputs: at most kPermSmall ids (vx_perm_small.cuh) --------

__global__ void __launch_bounds__(256) permute_small_kernel(
    const int32_t* __restrict__ ids, int P, int E, int shared_items, int k_div,
    const int32_t* __restrict__ src_map, int32_t* __restrict__ order,
    int32_t* __restrict__ inverse, int32_t* __restrict__ offsets, int32_t* __restrict__ active,
    int32_t* __restrict__ n_active, int32_t* __restrict__ src_rows, int32_t* __restrict__ err,
    int item_chunk, int32_t* __restrict__ items, int32_t* __restrict__ n_items) {
  chain_begin();
  PermSmallArgs a{E, shared_items, k_div, item_chunk, src_map, order, inverse, offsets, active,
                  n_active, src_rows, err, items, n_items};
  perm_small(a, ids, P);
}

// ---- prefill-sized inputs: slices of perm_slice(P) ids ----------------------

// Slices of 1,024 ids (one scatter chunk per CTA) up to 262,144 ids, then
// the smallest multiple of 1,024 that keeps the count at most 256: enough
// CTAs to cover the GPU at prefill sizes, and few enough slices for the
// scan's per-expert walk over them.
constexpr int64_t kPermMultiMin = 16384;

static int64_t perm_slice(int64_t P) {
  const int64_t unit = kPermThreads;
  const int64_t mult = (P + unit * 256 - 1) / (unit * 256);
  return unit * (mult > 1 ? mult : 1);
}

int64_t permute_scratch_ints(int64_t P, int E) {
  if (P <= kPermMultiMin) return 0;
  return ((P + perm_slice(P) - 1) / perm_slice(P)) * int64_t(E);
}

__global__ void __launch_bounds__(kPermThreads) permute_count_kernel(const int32_t* __restrict__ ids,
                                                                     int64_t P, int64_t slice, int E,
                                                                     int32_t* __restrict__ blk,
                                                                     int32_t* __restrict__ err) {
  chain_begin();
  extern __shared__ int counts[];
  __shared__ int s_bad;
  for (int e = threadIdx.x; e < E; e += kPermThreads) counts[e] = 0;
  if (threadIdx.x == 0) s_bad = 0;
  __syncthreads();
  const int64_t lo = int64_t(blockIdx.x) * slice;
  const int64_t hi = lo + slice < P ? lo + slice : P;
  const int bad = perm_count(ids, lo, hi, E, counts, &s_bad);
  for (int e = threadIdx.x; e < E; e += kPermThreads) blk[int64_t(blockIdx.x) * E + e] = counts[e];
  if (threadIdx.x == 0 && err && bad) atomicAdd(err, bad);
}

// One CTA: totals per expert, offsets and items, then each slice's starting
// position per expert (earlier slices first).
__global__ void __launch_bounds__(kPermThreads) permute_scan_kernel(
    int nb, int E, int shared_items, int32_t* __restrict__ blk, int32_t* __restrict__ offsets,
    int32_t* __restrict__ active, int32_t* __restrict__ n_active, int32_t* __restrict__ src_rows,
    int item_chunk, int32_t* __restrict__ items, int32_t* __restrict__ n_items) {
  chain_begin();
  extern __shared__ int smem[];
  int* counts = smem;           // [E]
  int* base = counts + E;       // [E]
  __shared__ int warp_tot[32];
  for (int e = threadIdx.x; e < E; e += kPermThreads) {
    int run = 0;
    for (int b = 0; b < nb; ++b) {
      const int c = blk[int64_t(b) * E + e];
      blk[int64_t(b) * E + e] = run;      // start of slice b inside expert e's run
      run += c;
    }
    counts[e] = run;
  }
  __syncthreads();
  perm_offsets(E, shared_items, counts, base, warp_tot, offsets, active, n_active, src_rows, item_chunk,
               items, n_items);
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += kPermThreads)
    for (int b = 0; b < nb; ++b) blk[int64_t(b) * E + e] += base[e];
}

__global__ void __launch_bounds__(kPermThreads) permute_scatter_kernel(
    const int32_t* __restrict__ ids, int64_t P, int64_t slice, int E, int k_div,
    const int32_t* __restrict__ src_map, const int32_t* __restrict__ blk, int32_t* __restrict__ order,
    int32_t* __restrict__ inverse, int32_t* __restrict__ src_rows) {
  chain_begin();
  extern __shared__ int smem[];
  int* running = smem;          // [E]
  int* hist = running + E;      // [kPermWarps][E]
  for (int e = threadIdx.x; e < E; e += kPermThreads) running[e] = blk[int64_t(blockIdx.x) * E + e];
  for (int i = threadIdx.x; i < kPermWarps * E; i += kPermThreads) hist[i] = 0;
  __syncthreads();
  const int64_t lo = int64_t(blockIdx.x) * slice;
  const int64_t hi = lo + slice < P ? lo + slice : P;
  perm_scatter(ids, lo, hi, E, k_div, src_map, running, hist, order, inverse, src_rows);
}

static cudaError_t set_smem(const void* fn, size_t smem) {
  if (smem <= 48 * 1024) return cudaSuccess;
  return cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
}

cudaError_t launch_permute(const int32_t* ids, int64_t P, int E, int shared_items, int k_div,
                           const int32_t* src_map, int32_t* order, int32_t* inverse,
                           int32_t* offsets, int32_t* active, int32_t* n_active,
                           int32_t* src_rows, int32_t* err, int item_chunk, int32_t* items,
                           int32_t* n_items, int32_t* blk, cudaStream_t st) {
  if (P <= kPermSmall && E <= kPermSmallMaxE)
    return launch_chained(permute_small_kernel, dim3(1), dim3(256), 0, st, ids, int(P), E, shared_items, k_div,
                          src_map, order, inverse, offsets, active, n_active, src_rows, err, item_chunk, items,
                          n_items);
  if (P <= kPermMultiMin || blk == nullptr) {
    const size_t smem = size_t(E) * (2 + kPermWarps) * sizeof(int);
    cudaError_t e = set_smem(reinterpret_cast<const void*>(permute_kernel), smem);
    if (e != cudaSuccess) return e;
    return launch_chained(permute_kernel, dim3(1), dim3(kPermThreads), smem, st, ids, int(P), E,
                          shared_items, k_div, src_map, order, inverse, offsets, active, n_active,
                          src_rows, err, item_chunk, items, n_items);
  }
  const int64_t slice = perm_slice(P);
  const int nb = int((P + slice - 1) / slice);
  cudaError_t e = launch_chained(permute_count_kernel, dim3(nb), dim3(kPermThreads),
                                 size_t(E) * sizeof(int), st, ids, P, slice, E, blk, err);
  if (e != cudaSuccess) return e;
  e = launch_chained(permute_scan_kernel, dim3(1), dim3(kPermThreads), size_t(E) * 2 * sizeof(int), st,
                     nb, E, shared_items, blk, offsets, active, n_active, src_rows, item_chunk, items,
                     n_items);
  if (e != cudaSuccess) return e;
  const size_t smem = size_t(E) * (1 + kPermWarps) * sizeof(int);
  e = set_smem(reinterpret_cast<const void*>(permute_scatter_kernel), smem);
  if (e != cudaSuccess) return e;
  return launch_chained(permute_scatter_kernel, dim3(nb), dim3(kPermThreads), smem, st, ids, P, slice, E,
                        k_div, src_map, blk, order, inverse, src_rows);
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
