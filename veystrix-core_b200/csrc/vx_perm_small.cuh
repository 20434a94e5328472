// Stable expert sort of a decode-sized id list (at most kPermSmall ids) by
// one 256-thread CTA: the same outputs as permute_kernel in vx_permute.cu
// (order, inverse, run offsets, active experts, work items, x rows).
#pragma once

#include "vx_common.cuh"
#include "vx_launch.h"

namespace vx {

// ---- decode-sized inputs: at most kPermSmall ids ---------------------------
// The same outputs as permute_kernel from one 256-thread CTA.  Ids are taken
// in rounds of 256 in index order (thread t holds id 256r + t of round r);
// an id's sorted position is its expert's run start, plus the equal ids of
// earlier rounds (a running count per expert), plus the equal ids of lower
// warps in the round (per-warp 16-bit counts tagged with the round, so a
// stale count of an earlier round reads as zero), plus its rank among equal
// lanes of its warp (peer_mask: one ballot per key bit).  The run offsets,
// the active list and the work items (each run cut into pieces of at most
// item_chunk positions, in expert order) come from the per-expert counts and
// one block scan of the three running totals.
constexpr int kPermSmallRounds = kPermSmall / 256;

// Lanes of the warp holding the same key as this lane, for keys in
// [-1, 1024): one ballot per bit (11 bits; -1 differs from every valid key in
// bit 10).  The same set as __match_any_sync, without its per-distinct-value
// cost when all 32 keys differ.
VX_DEVICE unsigned peer_mask(int key) {
  unsigned peers = 0xFFFFFFFFu;
#pragma unroll
  for (int b = 0; b < 11; ++b) {
    const bool bit = (key >> b) & 1;
    const unsigned v = __ballot_sync(0xFFFFFFFFu, bit);
    peers &= bit ? v : ~v;
  }
  return peers;
}

// Exclusive scan of one value per thread over a 256-thread CTA; *total gets
// the sum (valid on every thread after the call).
template <class V>
VX_DEVICE V scan256(V v, V* warp_tot, V* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  V inc = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const V n = __shfl_up_sync(0xFFFFFFFFu, inc, o);
    if (lane >= o) inc += n;
  }
  __syncthreads();   // warp_tot free from a previous call
  if (lane == 31) warp_tot[warp] = inc;
  __syncthreads();
  V before = 0, all = 0;
#pragma unroll
  for (int w = 0; w < 8; ++w) {
    const V t = warp_tot[w];
    before += w < warp ? t : V(0);
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
  __shared__ int s_cnt[kPermSmallMaxE];                    // ids per expert
  __shared__ int s_run[kPermSmallMaxE];                    // next position of each run
  __shared__ __align__(16) uint16_t s_hist[8][kPermSmallMaxE];   // (round + 1) << 8 | count
  __shared__ uint64_t warp_tot64[8];
  __shared__ int s_bad;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  for (int e = tid; e < E; e += 256) s_cnt[e] = 0;
  // only rows of warps below the last warp holding ids are ever read
  const int hist_rows = min(7, (min(P, 256) + 31) / 32 - 1);
  for (int w = 0; w < hist_rows; ++w)
    for (int e = tid; e < E; e += 256) s_hist[w][e] = 0;
  if (tid == 0) s_bad = 0;
  __syncthreads();
  int key[kPermSmallRounds];
  int nbad = 0;
  // all loads first (one memory round trip), then the counts
#pragma unroll
  for (int r = 0; r < kPermSmallRounds; ++r) {
    const int i = 256 * r + tid;
    key[r] = i < P ? __ldcg(ids + i) : -1;   // may have been written earlier in the same kernel
  }
#pragma unroll
  for (int r = 0; r < kPermSmallRounds; ++r) {
    const int i = 256 * r + tid;
    if (i >= P) continue;
    if (key[r] >= 0 && key[r] < E) {
      atomicAdd(&s_cnt[key[r]], 1);
    } else {
      key[r] = -1;
      inverse[i] = -1;
      ++nbad;
    }
  }
  if (nbad) atomicAdd(&s_bad, nbad);
  __syncthreads();

  // run offsets, active experts and work items: each thread takes a
  // contiguous block of E/256 experts; one scan carries the running counts
  // of active experts (bits 0-15), items (16-31) and routes (32-47), each at
  // most kPermSmall
  const int per = (E + 255) / 256, e0 = tid * per;
  uint64_t local = 0;
  for (int j = 0; j < per; ++j)
    if (e0 + j < E) {
      const uint64_t c = uint64_t(s_cnt[e0 + j]);
      if (c) local += 1u | (((c + item_chunk - 1) / item_chunk) << 16) | (c << 32);
    }
  uint64_t all;
  const uint64_t ex = scan256<uint64_t>(local, warp_tot64, &all);
  int run = int(ex >> 32) & 0xFFFF, ai = int(ex) & 0xFFFF, ii = int(ex >> 16) & 0xFFFF;
  const int routed = int(all >> 32) & 0xFFFF, n_act = int(all) & 0xFFFF, n_it = int(all >> 16) & 0xFFFF;
  for (int j = 0; j < per; ++j) {
    const int e = e0 + j;
    if (e >= E) break;
    const int c = s_cnt[e];
    s_run[e] = run;
    offsets[e] = run;
    if (c) {
      active[ai++] = e;
      if (items)
        for (int q = 0; q < c; q += item_chunk, ++ii) {
          int32_t* it = items + 3 * ii;
          it[0] = e;
          it[1] = run + q;
          it[2] = min(item_chunk, c - q);
        }
    }
    run += c;
  }
  const int sh_items = shared_items > 0 ? (shared_items + item_chunk - 1) / item_chunk : 0;
  if (tid == 0) {
    offsets[E] = routed;
    if (shared_items >= 0) offsets[E + 1] = routed + shared_items;
    if (err && s_bad) atomicAdd(err, s_bad);
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
  __syncthreads();

  // stable position of each valid id, one round of 256 ids at a time
  static_assert(kPermSmallMaxE <= 1024, "peer_mask covers 10-bit keys");
#pragma unroll 1
  for (int r = 0; r < kPermSmallRounds && 256 * r < P; ++r) {
    const int i = 256 * r + tid;
    int kr = key[0];
    if (r == 1) kr = key[1];
    if (r == 2) kr = key[2];
    if (r == 3) kr = key[3];
    const unsigned tag = unsigned(r + 1) << 8;
    const unsigned peers = peer_mask(kr);
    const int rank = __popc(peers & ((1u << lane) - 1u));
    const bool leader = (__ffs(peers) - 1) == lane;
    if (kr >= 0 && leader) s_hist[warp][kr] = uint16_t(tag | __popc(peers));
    __syncthreads();   // this round's counts are in; the previous round's runs advanced
    if (kr >= 0) {
      int pos = s_run[kr] + rank;
      for (int w = 0; w < warp; ++w) {
        const unsigned h = s_hist[w][kr];
        pos += (h & 0xFF00u) == tag ? int(h & 0xFFu) : 0;
      }
      order[pos] = i;
      inverse[i] = pos;
      if (src_rows) src_rows[pos] = src_map ? src_map[i] : i / k_div;
    }
    __syncthreads();   // s_run and s_hist read before they change
    if (kr >= 0 && leader) atomicAdd(&s_run[kr], __popc(peers));
  }
}

}  // namespace vx
