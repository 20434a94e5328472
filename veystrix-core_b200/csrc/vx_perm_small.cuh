// Stable expert sort of a decode-sized id list (at most kPermSmall ids) by
// one 256-thread CTA: the same outputs as permute_kernel in vx_permute.cu
// (order, inverse, run offsets, active experts, work items, x rows).
#pragma once

#include "vx_common.cuh"
#include "vx_launch.h"

namespace vx {

// ---- decode-sized inputs: at most kPermSmall ids ---------------------------
// The same outputs as permute_kernel from one 256-thread CTA with no
// per-expert histogram: an id's position is the number of valid ids below it
// plus the equal ids before it (a stable counting rank over at most 256
// ids), the run offsets come from per-expert counts and one block scan, and
// the active list and work items from run starts found in sorted order.

// Exclusive scan of one int per thread over a 256-thread CTA; *total gets
// the sum (valid on every thread after the call).
VX_DEVICE int scan256(int v, int* warp_tot, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int inc = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int n = __shfl_up_sync(0xFFFFFFFFu, inc, o);
    if (lane >= o) inc += n;
  }
  __syncthreads();   // warp_tot free from a previous call
  if (lane == 31) warp_tot[warp] = inc;
  __syncthreads();
  int before = 0, all = 0;
#pragma unroll
  for (int w = 0; w < 8; ++w) {
    const int t = warp_tot[w];
    before += w < warp ? t : 0;
    all += t;
  }
  *total = all;
  return before + inc - v;
}

// The permutation of ids[0..P) by one 256-thread CTA (every thread calls
// it); used by permute_small_kernel and by the fused router's last CTA.
VX_DEVICE void perm_small(const PermSmallArgs& a, const int32_t* ids, int P) {
  const int E = a.E, shared_items = a.shared_items, k_div = a.k_div, item_chunk = a.item_chunk;
  const int32_t* src_map = a.src_map;
  int32_t *order = a.order, *inverse = a.inverse, *offsets = a.offsets, *active = a.active;
  int32_t *n_active = a.n_active, *src_rows = a.src_rows, *err = a.err, *items = a.items;
  int32_t* n_items = a.n_items;
  __shared__ int s_key[kPermSmall];
  __shared__ int s_cnt[kPermSmallMaxE];
  __shared__ int s_off[kPermSmallMaxE];
  __shared__ int s_sorted[kPermSmall];   // expert of each sorted position
  __shared__ int warp_tot[8];
  const int tid = threadIdx.x;
  for (int e = tid; e < E; e += 256) s_cnt[e] = 0;
  int key = 0x7FFFFFFF;
  bool valid = false;
  if (tid < P) {
    const int id = __ldcg(ids + tid);   // may have been written earlier in the same kernel
    valid = id >= 0 && id < E;
    if (valid) key = id;
    else inverse[tid] = -1;
  }
  s_key[tid] = key;
  const int bad = __syncthreads_count(tid < P && !valid);
  if (valid) atomicAdd(&s_cnt[key], 1);
  __syncthreads();

  // run offsets: each thread scans a contiguous block of E/256 experts
  const int per = (E + 255) / 256, e0 = tid * per;
  int local = 0;
  for (int j = 0; j < per; ++j)
    if (e0 + j < E) local += s_cnt[e0 + j];
  int routed;
  int run = scan256(local, warp_tot, &routed);
  for (int j = 0; j < per; ++j)
    if (e0 + j < E) {
      s_off[e0 + j] = run;
      offsets[e0 + j] = run;
      run += s_cnt[e0 + j];
    }
  if (tid == 0) {
    offsets[E] = routed;
    if (shared_items >= 0) offsets[E + 1] = routed + shared_items;
    if (err && bad) atomicAdd(err, bad);
  }
  __syncthreads();

  // stable position of each valid id
  if (valid) {
    int r = s_off[key];
    for (int j = 0; j < tid; ++j) r += s_key[j] == key;
    order[r] = tid;
    inverse[tid] = r;
    s_sorted[r] = key;
    if (src_rows) src_rows[r] = src_map ? src_map[tid] : tid / k_div;
  }
  __syncthreads();

  // active experts and items, from the runs in sorted order
  const bool in = tid < routed;
  const int ek = in ? s_sorted[tid] : 0;
  const bool starts = in && (tid == 0 || s_sorted[tid - 1] != ek);
  const bool istart = in && ((tid - s_off[ek]) % item_chunk == 0);
  int n_act, n_it;
  const int ai = scan256(starts ? 1 : 0, warp_tot, &n_act);
  const int ii = scan256(istart ? 1 : 0, warp_tot, &n_it);
  if (starts) active[ai] = ek;
  if (items && istart) {
    int32_t* it = items + 3 * ii;
    it[0] = ek;
    it[1] = tid;
    it[2] = min(item_chunk, s_off[ek] + s_cnt[ek] - tid);
  }
  const int sh_items = shared_items > 0 ? (shared_items + item_chunk - 1) / item_chunk : 0;
  if (tid == 0) {
    if (shared_items > 0) active[n_act] = E;
    *n_active = n_act + (shared_items > 0 ? 1 : 0);
    if (items) *n_items = n_it + sh_items;
  }
  if (items)
    for (int j = tid; j < sh_items; j += 256) {
      int32_t* it = items + 3 * (n_it + j);
      it[0] = E;
      it[1] = routed + j * item_chunk;
      it[2] = min(item_chunk, shared_items - j * item_chunk);
    }
  if (src_rows)
    for (int t = tid; t < shared_items; t += 256) src_rows[routed + t] = t;
}


}  // namespace vx
