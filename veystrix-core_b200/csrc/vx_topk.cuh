// Softmax + top-k + renorm of one token's bf16 router logits, one warp per
// token (models/flashnext/adaptive_topk.py:59-65, :257-262; compiled.py:
// 60-70).  Shared by the router kernels and the single-launch decode kernel.
#pragma once

#include "vx_common.cuh"

namespace vx {

// ---- softmax + top-k + renorm: one warp per token --------------------------
// Register-only: lane r keeps the r-th selection.  The selection sum runs in
// slot order on every lane, as the reference's mass reduction does.
//
// Selection order: larger logit first, the smaller expert id among equal
// logits.  Each candidate is one 32-bit key - the bf16 logit mapped to an
// order-preserving unsigned 16-bit code (-0 folded onto +0, so zeros tie as
// equal floats do) above 0xFFFF - id - so a round of the selection is one
// warp-wide unsigned max (redux) plus a lane-local refresh.
constexpr int kMaxK = 32;

VX_DEVICE uint32_t logit_key(uint16_t b, int e) {
  if ((b & 0x7FFFu) == 0) b = 0;                                   // -0 -> +0
  if ((b & 0x7FFFu) > 0x7F80u) return 0u;                          // NaN: never selected
  const uint32_t ord = (b & 0x8000u) ? (~uint32_t(b) & 0xFFFFu) : (uint32_t(b) | 0x8000u);
  return (ord << 16) | (0xFFFFu - uint32_t(e));
}

VX_DEVICE float key_logit(uint32_t key) {
  const uint32_t ord = key >> 16;
  const uint32_t b = (ord & 0x8000u) ? (ord & 0x7FFFu) : (~ord & 0xFFFFu);
  return bf16_to_f32(uint16_t(b));
}

// Adaptive top-k (models/flashnext/adaptive_topk.py:44-51, :107-118,
// :224-233): a token keeps the smallest number of its leading slots whose
// share of its top-k probability mass reaches keep_mass - the running sum of
// p_r / sum(p), in double precision and slot order, as the reference's
// Python loop computes it - and at least keep_min (clamped to 1..k).
// keep_mass outside (0, 1) keeps every slot.  Lane r holds slot r's
// probability; every lane returns the same count.
__device__ __forceinline__ int topk_keep(float my_p, int k, double keep_mass, int keep_min) {
  if (!(keep_mass > 0.0 && keep_mass < 1.0)) return k;
  double total = 0.0;
  for (int r = 0; r < k; ++r) total += double(__shfl_sync(0xFFFFFFFFu, my_p, r));
  double acc = 0.0;
  int keep = k;
  for (int r = 0; r < k; ++r) {
    acc += double(__shfl_sync(0xFFFFFFFFu, my_p, r)) / total;
    if (acc >= keep_mass) {
      keep = r + 1;
      break;
    }
  }
  const int lo = keep_min < 1 ? 1 : (keep_min > k ? k : keep_min);
  return keep > lo ? keep : lo;
}

// Lane r < k gets the r-th largest of the warp's keys (0 once they run
// out); `key` is consumed.  Each lane sorts its PER keys in descending order
// (a bitonic network in registers: independent compare-exchanges), then a
// round is one warp-wide max of the lanes' heads and a one-place shift of
// the owner's list.  Keys are unique (the id is part of the key), so a
// nonzero maximum has one owner; the selection and its order are those of
// repeatedly taking the largest remaining key.
template <int PER>
__device__ __forceinline__ uint32_t topk_pick(uint32_t (&key)[PER], int k) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int size = 2; size <= PER; size <<= 1)
#pragma unroll
    for (int stride = size >> 1; stride > 0; stride >>= 1)
#pragma unroll
      for (int i = 0; i < PER; ++i) {
        const int l = i ^ stride;
        if (l > i) {
          const bool desc = (i & size) == 0;
          const uint32_t x = key[i], y = key[l];
          key[i] = desc ? max(x, y) : min(x, y);
          key[l] = desc ? min(x, y) : max(x, y);
        }
      }
  uint32_t my_key = 0;
  for (int r = 0; r < k; ++r) {
    const uint32_t g = __reduce_max_sync(0xFFFFFFFFu, key[0]);
    if (lane == r) my_key = g;
    const bool own = key[0] == g;
#pragma unroll
    for (int j = 0; j + 1 < PER; ++j) key[j] = own ? key[j + 1] : key[j];
    key[PER - 1] = own ? 0u : key[PER - 1];
  }
  return my_key;
}

template <int PER, bool COHERENT>
__device__ __forceinline__ void topk_row(const uint16_t* lr, int E, int k, int32_t* inds, uint16_t* scores,
                                         uint16_t* weights, uint16_t* mass, double keep_mass = 0.0,
                                         int keep_min = 1) {
  const int lane = threadIdx.x & 31;
  // Lane owns experts lane*PER .. lane*PER+PER-1 and fetches them with one
  // or a few vector loads, all issued before any is used (a chain of 2-byte
  // loads waited on one by one cost microseconds).  Logits written by other
  // CTAs of the same launch are read past L1.
  const int e0 = lane * PER;
  uint32_t raw[PER / 2];
  constexpr int kVec = PER >= 8 ? 8 : 4;   // bf16 per vector load
  const bool vec = e0 + PER <= E && E % kVec == 0 && (reinterpret_cast<uintptr_t>(lr) & (2 * kVec - 1)) == 0;
  if (vec) {
    if constexpr (PER >= 8) {
      const uint4* p = reinterpret_cast<const uint4*>(lr + e0);
      uint4 q[PER / 8];
#pragma unroll
      for (int v = 0; v < PER / 8; ++v) q[v] = COHERENT ? __ldcg(p + v) : p[v];
#pragma unroll
      for (int v = 0; v < PER / 8; ++v) {
        raw[4 * v] = q[v].x;
        raw[4 * v + 1] = q[v].y;
        raw[4 * v + 2] = q[v].z;
        raw[4 * v + 3] = q[v].w;
      }
    } else {
      const uint2 q = COHERENT ? __ldcg(reinterpret_cast<const uint2*>(lr + e0))
                               : *reinterpret_cast<const uint2*>(lr + e0);
      raw[0] = q.x;
      raw[1] = q.y;
    }
  } else {
#pragma unroll
    for (int j = 0; j < PER; j += 2) {
      const uint32_t lo = e0 + j < E ? (COHERENT ? __ldcg(lr + e0 + j) : lr[e0 + j]) : 0u;
      const uint32_t hi = e0 + j + 1 < E ? (COHERENT ? __ldcg(lr + e0 + j + 1) : lr[e0 + j + 1]) : 0u;
      raw[j / 2] = lo | (hi << 16);
    }
  }
  uint32_t key[PER];
  float m = -INFINITY;
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    const int e = e0 + j;
    const uint16_t b = uint16_t(raw[j / 2] >> (16 * (j & 1)));
    key[j] = e < E ? logit_key(b, e) : 0u;
    if (e < E) m = fmaxf(m, bf16_to_f32(b));
  }
  m = warp_max(m);
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < PER; ++j)
    if (e0 + j < E) s += expf(__fsub_rn(key_logit(key[j]), m));
  s = warp_sum<32>(s);
  const float inv = __fdiv_rn(1.0f, s);

  const uint32_t my_key = topk_pick<PER>(key, k);
  int my_i = int(0xFFFFu - (my_key & 0xFFFFu));
  const float my_p = bf16r(__fmul_rn(expf(__fsub_rn(key_logit(my_key), m)), inv));
  float tot = 0.f;
  for (int r = 0; r < k; ++r) tot = __fadd_rn(tot, __shfl_sync(0xFFFFFFFFu, my_p, r));
  // adaptive top-k: slots past the token's keep count repeat slot 0's expert
  // with probability 0 (every slot is kept unless 0 < keep_mass < 1)
  const int keep = topk_keep(my_p, k, keep_mass, keep_min);
  const int id0 = __shfl_sync(0xFFFFFFFFu, my_i, 0);
  const float kept_p = lane < keep ? my_p : 0.f;
  if (lane >= keep) my_i = id0;
  float sel = tot;
  if (keep < k) {
    sel = 0.f;
    for (int r = 0; r < k; ++r) sel = __fadd_rn(sel, __shfl_sync(0xFFFFFFFFu, kept_p, r));
  }
  // mass and renorm (blend 1.0): norm = mass + 1.0*(selected - mass), in bf16.
  const float msum = bf16r(tot);
  const float diff = bf16r(__fsub_rn(bf16r(sel), msum));
  const float norm = bf16r(__fadd_rn(msum, bf16r(diff)));
  if (lane < k) {
    inds[lane] = my_i;
    if (scores) scores[lane] = f32_to_bf16(kept_p);
    weights[lane] = f32_to_bf16(bf16r(__fdiv_rn(kept_p, norm)));
  }
  if (mass && lane == 0) *mass = f32_to_bf16(msum);
}

}  // namespace vx

namespace vx {

// The same routing split in two, for callers that need the ids before the
// weights: topk_select writes the top-k ids of one token (lane r < k holds
// the r-th selection, the order and tie rule of topk_row); topk_weights later
// writes the renormalised weights of given ids with exactly topk_row's
// arithmetic (per-lane sums over the lane's PER experts, then the same warp
// butterfly), so both halves together reproduce topk_row bit for bit.
template <int PER, bool COHERENT>
__device__ __forceinline__ void topk_load(const uint16_t* lr, int E, uint32_t (&raw)[PER / 2]) {
  const int lane = threadIdx.x & 31;
  const int e0 = lane * PER;
  constexpr int kVec = PER >= 8 ? 8 : 4;
  const bool vec = e0 + PER <= E && E % kVec == 0 && (reinterpret_cast<uintptr_t>(lr) & (2 * kVec - 1)) == 0;
  if (vec) {
    if constexpr (PER >= 8) {
      const uint4* p = reinterpret_cast<const uint4*>(lr + e0);
      uint4 q[PER / 8];
#pragma unroll
      for (int v = 0; v < PER / 8; ++v) q[v] = COHERENT ? __ldcg(p + v) : p[v];
#pragma unroll
      for (int v = 0; v < PER / 8; ++v) {
        raw[4 * v] = q[v].x;
        raw[4 * v + 1] = q[v].y;
        raw[4 * v + 2] = q[v].z;
        raw[4 * v + 3] = q[v].w;
      }
    } else {
      const uint2 q = COHERENT ? __ldcg(reinterpret_cast<const uint2*>(lr + e0))
                               : *reinterpret_cast<const uint2*>(lr + e0);
      raw[0] = q.x;
      raw[1] = q.y;
    }
  } else {
#pragma unroll
    for (int j = 0; j < PER; j += 2) {
      const uint32_t lo = e0 + j < E ? (COHERENT ? __ldcg(lr + e0 + j) : lr[e0 + j]) : 0u;
      const uint32_t hi = e0 + j + 1 < E ? (COHERENT ? __ldcg(lr + e0 + j + 1) : lr[e0 + j + 1]) : 0u;
      raw[j / 2] = lo | (hi << 16);
    }
  }
}

template <int PER, bool COHERENT>
__device__ __forceinline__ void topk_select(const uint16_t* lr, int E, int k, int32_t* inds) {
  const int lane = threadIdx.x & 31;
  const int e0 = lane * PER;
  uint32_t raw[PER / 2];
  topk_load<PER, COHERENT>(lr, E, raw);
  uint32_t key[PER];
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    const int e = e0 + j;
    key[j] = e < E ? logit_key(uint16_t(raw[j / 2] >> (16 * (j & 1))), e) : 0u;
  }
  const uint32_t my_key = topk_pick<PER>(key, k);
  if (lane < k) inds[lane] = int(0xFFFFu - (my_key & 0xFFFFu));
}

// topk_select that also leaves each selected key (the order-preserving key
// of the selected logit and id; 0 past the candidates) in keys[r], for
// topk_weights_keys.
template <int PER, bool COHERENT>
__device__ __forceinline__ void topk_select_keys(const uint16_t* lr, int E, int k, int32_t* inds,
                                                 uint32_t* keys) {
  const int lane = threadIdx.x & 31;
  const int e0 = lane * PER;
  uint32_t raw[PER / 2];
  topk_load<PER, COHERENT>(lr, E, raw);
  uint32_t key[PER];
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    const int e = e0 + j;
    key[j] = e < E ? logit_key(uint16_t(raw[j / 2] >> (16 * (j & 1))), e) : 0u;
  }
  const uint32_t my_key = topk_pick<PER>(key, k);
  if (lane < k) {
    inds[lane] = int(0xFFFFu - (my_key & 0xFFFFu));
    keys[lane] = my_key;
  }
}

// topk_weights for the keys topk_select_keys left: the softmax statistics
// of the row first, then `wait()` (the keys' hand-over), then the weights.
// Bit for bit topk_weights of the same selection (its per-lane sums in the
// same order; the key it rebuilds from the reloaded logit is the selected
// key itself).
template <int PER, bool COHERENT, class Wait>
__device__ __forceinline__ void topk_weights_keys(const uint16_t* lr, int E, int k, const uint32_t* keys,
                                                  uint16_t* weights, Wait wait) {
  const int lane = threadIdx.x & 31;
  const int e0 = lane * PER;
  uint32_t raw[PER / 2];
  topk_load<PER, COHERENT>(lr, E, raw);
  float m = -INFINITY;
  uint32_t key[PER];
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    const int e = e0 + j;
    const uint16_t b = uint16_t(raw[j / 2] >> (16 * (j & 1)));
    key[j] = e < E ? logit_key(b, e) : 0u;
    if (e < E) m = fmaxf(m, bf16_to_f32(b));
  }
  m = warp_max(m);
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < PER; ++j)
    if (e0 + j < E) s += expf(__fsub_rn(key_logit(key[j]), m));
  s = warp_sum<32>(s);
  const float inv = __fdiv_rn(1.0f, s);
  wait();
  const uint32_t my_key = lane < k ? keys[lane] : 0u;
  const float my_p = bf16r(__fmul_rn(expf(__fsub_rn(key_logit(my_key), m)), inv));
  float tot = 0.f;
  for (int r = 0; r < k; ++r) tot = __fadd_rn(tot, __shfl_sync(0xFFFFFFFFu, my_p, r));
  const float msum = bf16r(tot);
  const float diff = bf16r(__fsub_rn(msum, msum));
  const float norm = bf16r(__fadd_rn(msum, bf16r(diff)));
  if (lane < k) weights[lane] = f32_to_bf16(bf16r(__fdiv_rn(my_p, norm)));
}

template <int PER, bool COHERENT>
__device__ __forceinline__ void topk_weights(const uint16_t* lr, int E, int k, const int32_t* inds,
                                             uint16_t* weights) {
  const int lane = threadIdx.x & 31;
  const int e0 = lane * PER;
  uint32_t raw[PER / 2];
  topk_load<PER, COHERENT>(lr, E, raw);
  uint32_t key[PER];
  float m = -INFINITY;
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    const int e = e0 + j;
    const uint16_t b = uint16_t(raw[j / 2] >> (16 * (j & 1)));
    key[j] = e < E ? logit_key(b, e) : 0u;
    if (e < E) m = fmaxf(m, bf16_to_f32(b));
  }
  m = warp_max(m);
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < PER; ++j)
    if (e0 + j < E) s += expf(__fsub_rn(key_logit(key[j]), m));
  s = warp_sum<32>(s);
  const float inv = __fdiv_rn(1.0f, s);
  // the selected expert's key, as topk_select held it (0 for an id out of range)
  const int my_i = lane < k ? inds[lane] : -1;
  const uint32_t my_key =
      (my_i >= 0 && my_i < E) ? logit_key(COHERENT ? __ldcg(lr + my_i) : lr[my_i], my_i) : 0u;
  const float my_p = bf16r(__fmul_rn(expf(__fsub_rn(key_logit(my_key), m)), inv));
  float tot = 0.f;
  for (int r = 0; r < k; ++r) tot = __fadd_rn(tot, __shfl_sync(0xFFFFFFFFu, my_p, r));
  const float msum = bf16r(tot);
  const float diff = bf16r(__fsub_rn(msum, msum));
  const float norm = bf16r(__fadd_rn(msum, bf16r(diff)));
  if (lane < k) weights[lane] = f32_to_bf16(bf16r(__fdiv_rn(my_p, norm)));
}

}  // namespace vx
