// C ABI of libvxmoe (declared in include/vxmoe.h): argument validation,
// workspace carving and the launch sequence of each entry point.  No entry
// point allocates device memory or synchronises the host.
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>

#include "vx_common.cuh"
#include "vx_launch.h"
#include "vx_profile.h"

#define VX_VERSION_STRING "vxmoe 0.1.0 (sm_100a)"

static thread_local char g_cuda_err[256] = "";

int vx_cuda_fail(cudaError_t e) {
  snprintf(g_cuda_err, sizeof(g_cuda_err), "%s: %s", cudaGetErrorName(e), cudaGetErrorString(e));
  return VX_ECUDA;
}

namespace vx {

int sm_count() {
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cache[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    cache[dev] = n;
  }
  return cache[dev];
}

bool chain_enabled(bool streaming) {
  static int v = -1;
  if (v < 0) {
    const char* s = getenv("VXMOE_PDL");
    v = (s && strcmp(s, "0") == 0) ? 0 : (s && strcmp(s, "1") == 0) ? 1 : 2;
  }
  return v == 1 || (v == 2 && !streaming);
}

// Carves 256-byte aligned pieces out of a caller workspace.  With a null
// base it only measures.
struct Carver {
  char* base;
  size_t off = 0;
  explicit Carver(void* b) : base(static_cast<char*>(b)) {}
  template <class T>
  T* take(size_t n) {
    off = (off + 255) & ~size_t(255);
    T* p = base ? reinterpret_cast<T*>(base + off) : nullptr;
    off += n * sizeof(T);
    return p;
  }
  size_t size() const { return (off + 255) & ~size_t(255); }
};

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

static int check_q4(const vx_q4* b, int experts, int out, int in, int group = 32) {
  if (!b || !b->w || !b->scales || !b->biases) return VX_EINVAL_SHAPE;
  if (b->group_size != group) return VX_EUNSUPPORTED;
  if ((experts >= 0 && b->experts != experts) || b->out != out || b->in != in) return VX_EINVAL_SHAPE;
  if (b->in <= 0 || b->in % group || b->out <= 0) return VX_EINVAL_SHAPE;
  if (!aligned16(b->w)) return VX_EINVAL_SHAPE;
  return VX_OK;
}

struct BlockDims {
  int E, d, k, I, Is;
  bool shared;
  const vx_moe_pool* pool = nullptr;
  int path = VX_PATH_AUTO;   // the weights' expert_path
};

static int check_tiles(const vx_q4_tiles& t, int experts, int out, int in, int nproj, int group) {
  if (!t.records || !aligned16(t.records)) return VX_EINVAL_SHAPE;
  if (t.experts != experts || t.out != out || t.in != in || t.nproj != nproj) return VX_EINVAL_SHAPE;
  if (t.group_size != group || (group != 32 && group != 64) || in % group) return VX_EUNSUPPORTED;
  if (t.tile_rows != 16 && !(nproj == 1 && t.tile_rows == 32)) return VX_EINVAL_SHAPE;
  return VX_OK;
}

static int check_pool(const vx_moe_pool* p, int E, int d, int I, int Is, bool shared) {
  int s;
  // a pool of slots holds `slots` experts' records, addressed through slot_of
  if (p->slot_of && (p->slots < 1 || !aligned16(p->slot_of))) return VX_EINVAL_SHAPE;
  const int nrec = p->slot_of ? p->slots : E;
  // every part of a pool shares one quant group (32, or 64 natively)
  const int group = p->gate_up.group_size;
  if ((s = check_tiles(p->gate_up, nrec, I, d, 2, group))) return s;
  if ((s = check_tiles(p->down, nrec, d, I, 1, group))) return s;
  if (shared) {
    if ((s = check_tiles(p->shared_gate_up, 1, Is, d, 2, group))) return s;
    if ((s = check_tiles(p->shared_down, 1, d, Is, 1, group))) return s;
    // one launch serves routed and shared rows: the same row tiling
    if (p->shared_down.tile_rows != p->down.tile_rows) return VX_EINVAL_SHAPE;
  }
  return VX_OK;
}

static int check_weights(const vx_moe_weights* W, bool need_router, BlockDims* dm) {
  if (!W) return VX_EINVAL_SHAPE;
  const int E = W->num_experts, d = W->hidden, k = W->top_k;
  if (E < 1 || E > 1024 || d <= 0 || d % 32 || k < 1 || k > 16 || k > E) return VX_EINVAL_SHAPE;
  const int I = W->gate.out;
  int s;
  // the banks' group: 32, or the pool's native 64 (the banks then give shapes only)
  const int gb = W->pool && W->pool->gate_up.group_size == 64 ? 64 : 32;
  if ((s = check_q4(&W->gate, E, I, d, gb))) return s;
  if ((s = check_q4(&W->up, E, I, d, gb))) return s;
  if ((s = check_q4(&W->down, E, d, I, gb))) return s;
  if (I % 32) return VX_EINVAL_SHAPE;
  if (need_router && (!W->router_w || !aligned16(W->router_w))) return VX_EINVAL_SHAPE;
  const bool shared = W->shared_gate.w != nullptr;
  int Is = 0;
  if (shared) {
    Is = W->shared_gate.out;
    if ((s = check_q4(&W->shared_gate, 1, Is, d, gb))) return s;
    if ((s = check_q4(&W->shared_up, 1, Is, d, gb))) return s;
    if ((s = check_q4(&W->shared_down, 1, d, Is, gb))) return s;
    if (Is % 32) return VX_EINVAL_SHAPE;
    if (need_router && (s = check_q4(&W->shared_expert_gate, 1, 1, d))) return s;
  }
  if (W->pool && (s = check_pool(W->pool, E, d, I, Is, shared))) return s;
  if (W->expert_path < VX_PATH_AUTO || W->expert_path > VX_PATH_GEMM) return VX_EINVAL_SHAPE;
  *dm = {E, d, k, I, Is, shared, W->pool, W->expert_path};
  return VX_OK;
}

// Scratch of the routed-expert pipeline for T tokens (P = T*k items plus
// the shared expert's T items).
struct ExpertScratch {
  int32_t *order, *inverse, *offsets, *active, *n_active, *src_rows, *err, *items, *n_items;
  int32_t* blk;              // per-slice counts of the multi-CTA permutation (prefill sizes)
  uint16_t *h, *yd, *xb;     // xb: x in B order (MLX-layout path)
  float* xs;                 // per-group sum(x) of the T input rows (MLX-layout path)
  unsigned char *act, *hrec; // activation records of x and of h (tiled-pool path)
  int64_t ldh, ldxs;
  int max_items;
};

// Which expert pipeline runs a batch.  Decode-sized batches (a few tokens per
// expert) stream the weights through the GEMV - from the tiled pool when the
// weights carry one; prefill-sized batches (on average at least four routed
// positions per expert) take the tcgen05 GEMM.  The weights' expert_path
// forces one side; so does VXMOE_EXPERT_PATH=gemv|gemm when it is AUTO.
enum ExpertPath { kPathGemvMlx = 0, kPathGemvTiled = 1, kPathGemm = 2 };

static int path_override() {
  static int v = -1;
  if (v < 0) {
    const char* s = getenv("VXMOE_EXPERT_PATH");
    v = (s && strcmp(s, "gemv") == 0) ? 1 : (s && strcmp(s, "gemm") == 0) ? 2 : 0;
  }
  return v;
}

static ExpertPath expert_path(int T, const BlockDims& dm) {
  const int o = dm.path != VX_PATH_AUTO ? dm.path : path_override();
  const bool gemm = o == VX_PATH_GEMM || (o == VX_PATH_AUTO && int64_t(T) * dm.k >= 4 * int64_t(dm.E));
  if (gemm) return kPathGemm;
  return dm.pool ? kPathGemvTiled : kPathGemvMlx;
}

// Whether a block call runs as the single cooperative decode launch
// (vx_decode.cu): the tiled pool on the GEMV side, at most kDecodeMaxT
// tokens, shapes the kernel covers.  VXMOE_DECODE=0 keeps the multi-kernel
// pipeline (router, expert GEMVs, combine) for every batch.
static bool decode_enabled() {
  static int v = -1;
  if (v < 0) {
    const char* s = getenv("VXMOE_DECODE");
    v = (s && strcmp(s, "0") == 0) ? 0 : 1;
  }
  return v == 1;
}

static bool use_decode(int T, const BlockDims& dm) {
  // an explicit VX_PATH_GEMV / VX_PATH_GEMM (weights or VXMOE_EXPERT_PATH)
  // selects the multi-kernel pipelines
  if (dm.path != VX_PATH_AUTO || path_override() != 0) return false;
  if (!dm.pool || !decode_enabled() || expert_path(T, dm) != kPathGemvTiled) return false;
  if (dm.shared && dm.Is != dm.pool->shared_gate_up.out) return false;
  // the single launch reads records with groups of 32; native G64 records
  // take the multi-kernel GEMV pipeline
  if (dm.pool->gate_up.group_size != 32) return false;
  return decode_supported(T, dm.E, dm.d, dm.k, dm.I, dm.shared ? dm.Is : 0, dm.pool->gate_up.tile_rows,
                          dm.pool->down.tile_rows);
}

// Scratch of the decode launch: logits, sg, the SwiGLU outputs h and the
// four words (error bits, dropped ids, two barrier counters) that one memset
// clears.
struct DecodeScratch {
  uint16_t *logits, *sg, *h;
  int32_t* words;
  int ldh, Pp;
};

static DecodeScratch carve_decode(Carver& c, int T, const BlockDims& dm) {
  DecodeScratch s;
  s.Pp = T * dm.k + (dm.shared ? T : 0);
  s.ldh = std::max(dm.I, dm.shared ? dm.Is : 0);
  s.words = c.take<int32_t>(4);
  s.logits = c.take<uint16_t>(int64_t(T) * dm.E);
  s.sg = c.take<uint16_t>(T);
  s.h = c.take<uint16_t>(int64_t(s.Pp) * s.ldh);
  return s;
}

// Words of s.err, cleared before each call's expert pipeline: [0] dropped
// ids, [1] pipeline timeouts, [2] [3] the task counters of the gate/up and
// down GEMVs (tasks handed out dynamically).
constexpr int kErrWords = 4;

// extra_zeroed: ints placed right after s.err, so that one memset clears
// both (the block call keeps the router's arrival counters there).
static ExpertScratch carve_experts(Carver& c, int T, const BlockDims& dm, int extra_zeroed = 0) {
  const int64_t P = int64_t(T) * dm.k, Ts = dm.shared ? T : 0;
  const ExpertPath path = expert_path(T, dm);
  ExpertScratch s;
  s.order = c.take<int32_t>(P);
  s.inverse = c.take<int32_t>(P);
  s.offsets = c.take<int32_t>(dm.E + 2);
  s.active = c.take<int32_t>(dm.E + 1);
  s.n_active = c.take<int32_t>(1);
  s.src_rows = c.take<int32_t>(P + Ts);
  s.err = c.take<int32_t>(kErrWords + extra_zeroed);
  s.max_items = max_items_bound(P, dm.E, int(Ts));
  s.items = c.take<int32_t>(3 * int64_t(s.max_items));
  s.n_items = c.take<int32_t>(1);
  s.blk = c.take<int32_t>(permute_scratch_ints(P, dm.E));
  s.ldh = std::max(dm.I, dm.Is);
  s.yd = c.take<uint16_t>((P + Ts) * dm.d);
  s.ldxs = xsum_stride(dm.d);
  s.h = s.xb = nullptr;
  s.xs = nullptr;
  s.act = s.hrec = nullptr;
  if (path == kPathGemm) {
    s.h = c.take<uint16_t>((P + Ts) * s.ldh);
    s.xb = c.take<uint16_t>((P + Ts) * dm.d);   // x gathered into sorted order
  } else if (path == kPathGemvTiled) {
    s.act = c.take<unsigned char>(act_record_bytes(dm.d, P + Ts));
    s.h = c.take<uint16_t>((P + Ts) * s.ldh);
    s.hrec = c.take<unsigned char>(act_record_bytes(int(s.ldh), P + Ts));
  } else {
    s.h = c.take<uint16_t>((P + Ts) * s.ldh);
    s.xb = c.take<uint16_t>(int64_t(T) * dm.d);
    s.xs = c.take<float>(int64_t(T) * s.ldxs);
  }
  return s;
}

// permute -> gate/up + SwiGLU -> down, leaving sorted bf16 outputs in s.yd.
// Positions per work item of each pipeline.
static int item_chunk(ExpertPath path, const BlockDims& dm) {
  return path == kPathGemm ? (dm.pool ? kPoolGemmItemChunk : kGemmItemChunk)
         : path == kPathGemvTiled ? kTiledItemChunk : kItemChunk;
}

// err_zeroed: the caller cleared s.err earlier on the stream, so no memset
// node breaks the chain of programmatically serialised kernels.  permuted:
// the router already sorted the routes into s (decode-sized batches).
static int run_experts(const uint16_t* x, int T, const int32_t* routes, const vx_moe_weights* W,
                       const BlockDims& dm, const ExpertScratch& s, cudaStream_t st,
                       bool err_zeroed = false, bool permuted = false) {
  const int64_t P = int64_t(T) * dm.k;
  const int Ts = dm.shared ? T : 0;
  cudaError_t e = cudaSuccess;
  if (!err_zeroed) {
    e = cudaMemsetAsync(s.err, 0, kErrWords * sizeof(int32_t), st);
    if (e != cudaSuccess) return vx_cuda_fail(e);
  }
  const ExpertPath path = expert_path(T, dm);
  if (!permuted) {
    e = launch_permute(routes, P, dm.E, Ts, dm.k, nullptr, s.order, s.inverse, s.offsets, s.active,
                       s.n_active, s.src_rows, s.err, item_chunk(path, dm), s.items, s.n_items, s.blk, st);
    if (e != cudaSuccess) return vx_cuda_fail(e);
  }
  if (path == kPathGemm) {
    e = launch_gather_border(x, dm.d, dm.d, s.src_rows, s.offsets + dm.E + 1, P + Ts, s.xb, st);
    if (e != cudaSuccess) return vx_cuda_fail(e);
    profile_mark(st, "permute");
    if (dm.pool) {
      // persistent kernel over the tiled pool's records
      const vx_moe_pool& pl = *dm.pool;
      PoolGemmArgs a{};
      a.err = s.err + 1;
      a.rec_b = static_cast<const unsigned char*>(pl.gate_up.records);
      a.stride_b = tile_pool_bytes(1, dm.I, dm.d, 2, pl.gate_up.tile_rows, pl.gate_up.group_size);
      a.slot_of = pl.slot_of;
      a.slots = pl.slots;
      a.group = pl.gate_up.group_size;
      a.rec_s = dm.shared ? static_cast<const unsigned char*>(pl.shared_gate_up.records) : nullptr;
      a.N_b = dm.I;
      a.N_s = dm.Is;
      a.K_b = a.K_s = dm.d;
      a.tile_rows = pl.gate_up.tile_rows;
      a.E = dm.E;
      a.items = s.items;
      a.n_items = s.n_items;
      a.out = s.h;
      a.ldo = s.ldh;
      e = launch_gemm_pool(true, a, s.xb, P + Ts, dm.d, s.max_items, st);
      if (e != cudaSuccess) return vx_cuda_fail(e);
      profile_mark(st, "gate_up_swiglu");
      PoolGemmArgs b{};
      b.err = s.err + 1;
      b.rec_b = static_cast<const unsigned char*>(pl.down.records);
      b.stride_b = tile_pool_bytes(1, dm.d, dm.I, 1, pl.down.tile_rows, pl.down.group_size);
      b.slot_of = pl.slot_of;
      b.slots = pl.slots;
      b.group = pl.down.group_size;
      b.rec_s = dm.shared ? static_cast<const unsigned char*>(pl.shared_down.records) : nullptr;
      b.N_b = b.N_s = dm.d;
      b.K_b = dm.I;
      b.K_s = dm.Is;
      b.tile_rows = pl.down.tile_rows;
      b.E = dm.E;
      b.items = s.items;
      b.n_items = s.n_items;
      b.out = s.yd;
      b.ldo = dm.d;
      e = launch_gemm_pool(false, b, s.h, P + Ts, s.ldh, s.max_items, st);
      if (e != cudaSuccess) return vx_cuda_fail(e);
      profile_mark(st, "down");
      return VX_OK;
    }
    GemmArgs a{};
    a.err = s.err + 1;
    a.b0 = W->gate;
    a.b1 = W->up;
    if (dm.shared) {
      a.s0 = W->shared_gate;
      a.s1 = W->shared_up;
    }
    a.E = dm.E;
    a.items = s.items;
    a.n_items = s.n_items;
    a.out = s.h;
    a.ldo = s.ldh;
    e = launch_gemm_tc(true, a, s.xb, P + Ts, dm.d, s.max_items, st);
    if (e != cudaSuccess) return vx_cuda_fail(e);
    profile_mark(st, "gate_up_swiglu");
    GemmArgs b{};
    b.err = s.err + 1;
    b.b0 = W->down;
    if (dm.shared) b.s0 = W->shared_down;
    b.E = dm.E;
    b.items = s.items;
    b.n_items = s.n_items;
    b.out = s.yd;
    b.ldo = dm.d;
    e = launch_gemm_tc(false, b, s.h, P + Ts, s.ldh, s.max_items, st);
    if (e != cudaSuccess) return vx_cuda_fail(e);
    profile_mark(st, "down");
    return VX_OK;
  }
  if (path == kPathGemvTiled) {
    // activation records of the sorted positions (valid count: offsets[E+1])
    e = launch_act_records(x, dm.d, dm.d, s.src_rows, s.offsets + dm.E + 1, P + Ts, s.act, st);
    // h records are built over ldh = max(I, Is) columns: when the routed and
    // shared widths differ, the narrower rows' columns up to ldh must read 0
    if (e == cudaSuccess && dm.shared && dm.I != dm.Is)
      e = cudaMemsetAsync(s.h, 0, size_t(P + Ts) * size_t(s.ldh) * sizeof(uint16_t), st);
  } else {
    e = launch_xprep(x, T, dm.d, s.xb, s.xs, s.ldxs, st);
  }
  if (e != cudaSuccess) return vx_cuda_fail(e);
  profile_mark(st, "permute");

  if (path == kPathGemvTiled) {
    const vx_moe_pool& pl = *dm.pool;
    TiledArgs a{};
    a.err = s.err + 1;
    a.rec_b = static_cast<const unsigned char*>(pl.gate_up.records);
    a.stride_b = tile_pool_bytes(1, dm.I, dm.d, 2, pl.gate_up.tile_rows, pl.gate_up.group_size);
    a.slot_of = pl.slot_of;
    a.slots = pl.slots;
    a.rec_s = dm.shared ? static_cast<const unsigned char*>(pl.shared_gate_up.records) : nullptr;
    a.N_b = dm.I;
    a.N_s = dm.Is;
    a.K_b = a.K_s = dm.d;
    a.E = dm.E;
    a.items = s.items;
    a.n_items = s.n_items;
    a.act = s.act;
    a.act_rows = P + Ts;
    a.out = s.h;
    a.ldo = s.ldh;
    a.task_ctr = s.err + 2;
    e = launch_gemv_tiled(true, pl.gate_up.tile_rows, a, s.max_items, int(s.ldh), st, pl.gate_up.group_size);
    if (e != cudaSuccess) return vx_cuda_fail(e);
    profile_mark(st, "gate_up_swiglu");
    e = launch_act_records(s.h, s.ldh, int(s.ldh), nullptr, s.offsets + dm.E + 1, P + Ts, s.hrec, st);
    if (e != cudaSuccess) return vx_cuda_fail(e);
    profile_mark(st, "h_records");

    TiledArgs b{};
    b.err = s.err + 1;
    b.rec_b = static_cast<const unsigned char*>(pl.down.records);
    b.stride_b = tile_pool_bytes(1, dm.d, dm.I, 1, pl.down.tile_rows, pl.down.group_size);
    b.slot_of = pl.slot_of;
    b.slots = pl.slots;
    b.rec_s = dm.shared ? static_cast<const unsigned char*>(pl.shared_down.records) : nullptr;
    b.N_b = b.N_s = dm.d;
    b.K_b = dm.I;
    b.K_s = dm.Is;
    b.E = dm.E;
    b.items = s.items;
    b.n_items = s.n_items;
    b.act = s.hrec;
    b.act_rows = P + Ts;
    b.task_ctr = s.err + 3;
    b.out = s.yd;
    b.ldo = dm.d;
    e = launch_gemv_tiled(false, pl.down.tile_rows, b, s.max_items, dm.d, st, pl.down.group_size);
    if (e != cudaSuccess) return vx_cuda_fail(e);
    profile_mark(st, "down");
    return VX_OK;
  }

  MmaArgs a{};
  a.b0 = W->gate;
  a.b1 = W->up;
  if (dm.shared) {
    a.s0 = W->shared_gate;
    a.s1 = W->shared_up;
  }
  a.E = dm.E;
  a.err = s.err + 1;
  a.items = s.items;
  a.n_items = s.n_items;
  a.src_rows = s.src_rows;
  a.dst_rows = nullptr;
  a.x = s.xb;
  a.ldx = dm.d;
  a.xsum = s.xs;
  a.ldxs = s.ldxs;
  a.out = s.h;
  a.ldo = s.ldh;
  e = launch_gemv_mma(true, a, s.max_items, int(s.ldh), st);
  if (e != cudaSuccess) return vx_cuda_fail(e);
  profile_mark(st, "gate_up_swiglu");

  MmaArgs b{};
  b.b0 = W->down;
  if (dm.shared) b.s0 = W->shared_down;
  b.E = dm.E;
  b.err = s.err + 1;
  b.items = s.items;
  b.n_items = s.n_items;
  b.src_rows = nullptr;
  b.dst_rows = nullptr;
  b.x = s.h;
  b.ldx = s.ldh;
  b.out = s.yd;
  b.ldo = dm.d;
  e = launch_gemv_mma(false, b, s.max_items, dm.d, st);
  if (e != cudaSuccess) return vx_cuda_fail(e);
  profile_mark(st, "down");
  return VX_OK;
}

struct RouterScratch {
  uint16_t* logits;
};

// The checks vx_moe_block makes before it looks at the workspace: the
// weights, the token count and the activation pointers.  VX_OK for a valid
// call (T == 0 included).
int block_args_status(const uint16_t* x, int T, const vx_moe_weights* W, const uint16_t* y) {
  BlockDims dm;
  int s = check_weights(W, true, &dm);
  if (s) return s;
  if (T < 0) return VX_EINVAL_SHAPE;
  if (T == 0) return VX_OK;
  if (!x || !y || !aligned16(x)) return VX_EINVAL_SHAPE;
  return VX_OK;
}

}  // namespace vx

using namespace vx;

extern "C" {

const char* vx_version(void) { return VX_VERSION_STRING; }

const char* vx_strerror(int status) {
  switch (status) {
    case VX_OK: return "ok";
    case VX_EINVAL_SHAPE: return "invalid shape or size";
    case VX_EINVAL_DTYPE: return "invalid dtype";
    case VX_EINVAL_INDEX: return "index out of range";
    case VX_ECUDA: return "CUDA error";
    case VX_ETIMEOUT: return "timed out";
    case VX_EWORKSPACE: return "workspace too small";
    case VX_EUNSUPPORTED: return "unsupported configuration";
    default: return "unknown status";
  }
}

const char* vx_last_cuda_error(void) { return g_cuda_err; }

size_t vx_q4_tiles_bytes_group(int32_t experts, int32_t out, int32_t in, int32_t nproj, int32_t tile_rows,
                               int32_t group_size) {
  if (group_size != 32 && group_size != 64) return 0;
  if (experts < 1 || out < 1 || in < group_size || in % group_size || (nproj != 1 && nproj != 2)) return 0;
  if (tile_rows != 16 && !(nproj == 1 && tile_rows == 32)) return 0;
  return size_t(tile_pool_bytes(experts, out, in, nproj, tile_rows, group_size));
}

size_t vx_q4_tiles_bytes(int32_t experts, int32_t out, int32_t in, int32_t nproj,
                         int32_t tile_rows) {
  return vx_q4_tiles_bytes_group(experts, out, in, nproj, tile_rows, 32);
}

int vx_q4_tile(const vx_q4* a, const vx_q4* b, int32_t nproj, int32_t tile_rows, void* records,
               size_t records_bytes, void* stream) {
  if (!a) return VX_EINVAL_SHAPE;
  // the records keep the banks' group: 32, or 64 natively
  const int group = a->group_size == 64 ? 64 : 32;
  int s = check_q4(a, -1, a->out, a->in, group);
  if (s) return s;
  if (nproj == 2) {
    if (!b) return VX_EINVAL_SHAPE;
    if ((s = check_q4(b, a->experts, a->out, a->in, group))) return s;
  }
  const size_t need = vx_q4_tiles_bytes_group(a->experts, a->out, a->in, nproj, tile_rows, group);
  if (need == 0) return VX_EINVAL_SHAPE;
  if (!records || !aligned16(records)) return VX_EINVAL_SHAPE;
  if (records_bytes < need) return VX_EWORKSPACE;
  cudaError_t e = launch_tile_pack(*a, nproj == 2 ? *b : *a, nproj, tile_rows, records,
                                   static_cast<cudaStream_t>(stream), group);
  return e == cudaSuccess ? VX_OK : vx_cuda_fail(e);
}

int vx_q4_dequant(const vx_q4* bank, int32_t expert, float* out, void* stream) {
  if (!bank || !out || !bank->w || !bank->scales || !bank->biases) return VX_EINVAL_SHAPE;
  if (bank->group_size <= 0 || bank->in % bank->group_size || bank->in % 8) return VX_EINVAL_SHAPE;
  if (expert < 0 || expert >= bank->experts) return VX_EINVAL_INDEX;
  cudaError_t e = launch_dequant(*bank, expert, out, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? VX_OK : vx_cuda_fail(e);
}

int vx_swiglu_bf16(const uint16_t* gate, const uint16_t* up, uint16_t* out, int64_t n,
                   void* stream) {
  if (n < 0 || (n > 0 && (!gate || !up || !out))) return VX_EINVAL_SHAPE;
  cudaError_t e = launch_swiglu(gate, up, out, n, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? VX_OK : vx_cuda_fail(e);
}

size_t vx_gather_qmm_workspace(int64_t B, int32_t M, int32_t experts, int64_t x_rows, int32_t K) {
  Carver c(nullptr);
  const int64_t n = B * M;
  c.take<uint16_t>(x_rows * K);                 // x in B order
  c.take<float>(x_rows * xsum_stride(K));       // sum(x) per group
  c.take<int32_t>(n);            // keys
  c.take<int32_t>(n);            // src_map
  c.take<int32_t>(n);            // order
  c.take<int32_t>(n);            // inverse
  c.take<int32_t>(experts + 2);  // offsets
  c.take<int32_t>(experts + 1);  // active
  c.take<int32_t>(1);            // n_active
  c.take<int32_t>(n);            // src_rows
  c.take<int32_t>(2);            // err
  c.take<int32_t>(3 * int64_t(max_items_bound(n, experts, 0)));  // items
  c.take<int32_t>(1);            // n_items
  return c.size();
}

int vx_gather_qmm(const uint16_t* x, int64_t x_rows, const vx_q4* w, const int32_t* lhs,
                  const int32_t* rhs, int64_t B, int32_t M, int32_t sorted_indices, uint16_t* out,
                  void* workspace, size_t workspace_bytes, void* stream) {
  (void)sorted_indices;
  if (!w || B < 0 || M < 1) return VX_EINVAL_SHAPE;
  int s = check_q4(w, w->experts, w->out, w->in);
  if (s) return s;
  if (w->experts < 1 || w->experts > 1024) return VX_EUNSUPPORTED;
  if (B * M > 0x7FFFFFFF) return VX_EUNSUPPORTED;
  if (B == 0) return VX_OK;
  if (!x || !rhs || !out || !aligned16(x)) return VX_EINVAL_SHAPE;
  if (x_rows < 0) return VX_EINVAL_SHAPE;
  if (workspace_bytes < vx_gather_qmm_workspace(B, M, w->experts, x_rows, w->in) || !workspace)
    return VX_EWORKSPACE;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t n = B * M;
  const int E = w->experts;
  Carver c(workspace);
  uint16_t* xb = c.take<uint16_t>(x_rows * w->in);
  const int64_t ldxs = xsum_stride(w->in);
  float* xs = c.take<float>(x_rows * ldxs);
  int32_t* keys = c.take<int32_t>(n);
  int32_t* src_map = c.take<int32_t>(n);
  int32_t* order = c.take<int32_t>(n);
  int32_t* inverse = c.take<int32_t>(n);
  int32_t* offsets = c.take<int32_t>(E + 2);
  int32_t* active = c.take<int32_t>(E + 1);
  int32_t* n_active = c.take<int32_t>(1);
  int32_t* src_rows = c.take<int32_t>(n);
  int32_t* err = c.take<int32_t>(2);
  const int max_items = max_items_bound(n, E, 0);
  int32_t* items = c.take<int32_t>(3 * int64_t(max_items));
  int32_t* n_items = c.take<int32_t>(1);
  cudaError_t e = cudaMemsetAsync(err, 0, 2 * sizeof(int32_t), st);
  if (e == cudaSuccess) e = launch_xprep(x, x_rows, w->in, xb, xs, ldxs, st);
  if (e == cudaSuccess) e = launch_gather_items(lhs, rhs, B, M, x_rows, keys, src_map, st);
  if (e == cudaSuccess)
    e = launch_permute(keys, n, E, 0, 1, src_map, order, inverse, offsets, active, n_active, src_rows,
                       err, kItemChunk, items, n_items, nullptr, st);
  if (e != cudaSuccess) return vx_cuda_fail(e);
  MmaArgs a{};
  a.b0 = *w;
  a.err = err + 1;
  a.E = E;
  a.items = items;
  a.n_items = n_items;
  a.src_rows = src_rows;
  a.dst_rows = order;
  a.x = xb;
  a.ldx = w->in;
  a.xsum = xs;
  a.ldxs = ldxs;
  a.out = out;
  a.ldo = w->out;
  e = launch_gemv_mma(false, a, max_items, w->out, st);
  return e == cudaSuccess ? VX_OK : vx_cuda_fail(e);
}

int vx_softmax_topk(const uint16_t* logits, int32_t T, int32_t E, int32_t k, int32_t* inds,
                    uint16_t* scores, uint16_t* weights, uint16_t* mass, void* stream) {
  if (T < 0 || E < 1 || E > 1024 || k < 1 || k > 16 || k > E) return VX_EINVAL_SHAPE;
  if (T == 0) return VX_OK;
  if (!logits || !inds || !weights) return VX_EINVAL_SHAPE;
  cudaError_t e = launch_softmax_topk(logits, T, E, k, inds, scores, weights, mass,
                                      static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? VX_OK : vx_cuda_fail(e);
}

size_t vx_router_workspace(int32_t T, const vx_moe_weights* W) {
  if (!W || T < 0) return 0;
  Carver c(nullptr);
  c.take<uint16_t>(int64_t(T) * W->num_experts);   // logits (when the caller passes none)
  c.take<int32_t>(router_counters(T));             // arrival counters of the fused router
  return c.size();
}

// Decode-sized batches: one launch - logits, top-k and renorm by the last CTA
// of each token block, and the shared-expert gate (vx_router.cu
// router_fused_kernel).  Prefill-sized batches: the tiled logits kernel and
// the softmax/top-k kernel (the same bits).
static int router_impl(const uint16_t* x, int T, const vx_moe_weights* W, const BlockDims& dm,
                       uint16_t* logits, int32_t* inds, uint16_t* weights, uint16_t* sg,
                       int32_t* counters, cudaStream_t st, const PermSmallArgs* perm = nullptr,
                       bool counters_zeroed = false) {
  profile_mark(st, "");
  const bool gate = sg && W->shared_expert_gate.w;
  cudaError_t e;
  if (!perm && router_tiled_fits(T, dm.d))   // prefill-sized batch: tiled logits, then top-k
    e = launch_router_tiled(x, T, W->router_w, dm.E, dm.d, dm.k, gate ? &W->shared_expert_gate : nullptr,
                            logits, inds, weights, gate ? sg : nullptr, W->router_bias, st, W->keep_mass,
                            W->keep_min);
  else
    e = launch_router_fused(x, T, W->router_w, dm.E, dm.d, dm.k, gate ? &W->shared_expert_gate : nullptr,
                            logits, inds, weights, gate ? sg : nullptr, counters, perm, W->router_bias, st,
                            counters_zeroed, W->keep_mass, W->keep_min);
  if (e != cudaSuccess) return vx_cuda_fail(e);
  profile_mark(st, "router");
  return VX_OK;
}

int vx_router(const uint16_t* x, int32_t T, const vx_moe_weights* W, uint16_t* logits,
              int32_t* inds, uint16_t* weights, uint16_t* sg, void* workspace,
              size_t workspace_bytes, void* stream) {
  // The router needs only the gate weights and the shared expert gate (an
  // expert-parallel rank holds just its shard of the expert banks).
  if (!W) return VX_EINVAL_SHAPE;
  BlockDims dm{W->num_experts, W->hidden, W->top_k, 0, 0, false};
  if (dm.E < 1 || dm.E > 1024 || dm.d <= 0 || dm.d % 32 || dm.k < 1 || dm.k > 16 || dm.k > dm.E)
    return VX_EINVAL_SHAPE;
  if (!W->router_w || !aligned16(W->router_w)) return VX_EINVAL_SHAPE;
  if (W->shared_expert_gate.w) {
    int s = check_q4(&W->shared_expert_gate, 1, 1, dm.d);
    if (s) return s;
  }
  if (T < 0) return VX_EINVAL_SHAPE;
  if (T == 0) return VX_OK;
  if (!x || !inds || !weights || !aligned16(x)) return VX_EINVAL_SHAPE;
  if (!workspace || workspace_bytes < vx_router_workspace(T, W)) return VX_EWORKSPACE;
  Carver c(workspace);
  uint16_t* lg = c.take<uint16_t>(int64_t(T) * dm.E);
  int32_t* counters = c.take<int32_t>(router_counters(T));
  if (!logits) logits = lg;
  return router_impl(x, T, W, dm, logits, inds, weights, sg, counters, static_cast<cudaStream_t>(stream));
}

size_t vx_permute_workspace(int64_t P, int32_t E) {
  Carver c(nullptr);
  c.take<int32_t>(E + 1);
  c.take<int32_t>(1);
  c.take<int32_t>(permute_scratch_ints(P, E));   // per-slice counts (large P)
  return c.size();
}

int vx_permute(const int32_t* ids, int64_t P, int32_t E, int32_t* order, int32_t* inverse,
               int32_t* offsets, int32_t* error_count, void* workspace, size_t workspace_bytes,
               void* stream) {
  if (P < 0 || P > 0x7FFFFFFF || E < 1 || E > 4096) return VX_EINVAL_SHAPE;
  if (!offsets) return VX_EINVAL_SHAPE;
  if (P > 0 && (!ids || !order || !inverse)) return VX_EINVAL_SHAPE;
  if (!workspace || workspace_bytes < vx_permute_workspace(P, E)) return VX_EWORKSPACE;
  Carver c(workspace);
  int32_t* active = c.take<int32_t>(E + 1);
  int32_t* n_active = c.take<int32_t>(1);
  int32_t* blk = c.take<int32_t>(permute_scratch_ints(P, E));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = launch_permute(ids, P, E, -1, 1, nullptr, order, inverse, offsets, active, n_active,
                                 nullptr, error_count, kItemChunk, nullptr, nullptr, blk, st);
  return e == cudaSuccess ? VX_OK : vx_cuda_fail(e);
}

size_t vx_moe_experts_workspace(int32_t T, const vx_moe_weights* W) {
  if (!W || T < 0) return 0;
  BlockDims dm{W->num_experts, W->hidden, W->top_k, W->gate.out, 0, false, W->pool,
               W->expert_path};
  Carver c(nullptr);
  carve_experts(c, T, dm);
  return c.size();
}

int vx_moe_experts(const uint16_t* x, int32_t T, const int32_t* routes, const uint16_t* scores,
                   const vx_moe_weights* W, const uint16_t* shared_y, const uint16_t* shared,
                   const uint16_t* shared_gate, uint16_t* out, void* workspace,
                   size_t workspace_bytes, void* stream) {
  BlockDims dm;
  int s = check_weights(W, false, &dm);
  if (s) return s;
  dm.shared = false;  // the executor takes the shared expert from its caller
  dm.Is = 0;
  if (T < 0) return VX_EINVAL_SHAPE;
  if ((shared == nullptr) != (shared_gate == nullptr)) return VX_EINVAL_SHAPE;
  if (shared_y && shared) return VX_EINVAL_SHAPE;
  if (T == 0) return VX_OK;
  if (!x || !routes || !out || !aligned16(x)) return VX_EINVAL_SHAPE;
  if (!workspace || workspace_bytes < vx_moe_experts_workspace(T, W)) return VX_EWORKSPACE;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  Carver c(workspace);
  ExpertScratch es = carve_experts(c, T, dm);
  profile_mark(st, "");
  s = run_experts(x, T, routes, W, dm, es, st);
  if (s) return s;
  cudaError_t e;
  if (scores) {
    SharedMode mode = shared_y ? kSharedY : (shared ? kSharedParts : kSharedNone);
    e = launch_combine(es.yd, dm.d, es.inverse, scores, T, dm.k, dm.d, mode, es.offsets, dm.E,
                       nullptr, shared_y, shared, shared_gate, out, st);
  } else {
    e = launch_unpermute(es.yd, dm.d, es.inverse, T, dm.k, dm.d, out, st);
  }
  if (e != cudaSuccess) return vx_cuda_fail(e);
  profile_mark(st, scores ? "combine" : "unpermute");
  return VX_OK;
}

int vx_moe_experts_partial(const uint16_t* x, int32_t T, const int32_t* routes,
                           const uint16_t* scores, const vx_moe_weights* W, float* out,
                           void* workspace, size_t workspace_bytes, void* stream) {
  BlockDims dm;
  int s = check_weights(W, false, &dm);
  if (s) return s;
  dm.shared = false;
  dm.Is = 0;
  if (T < 0) return VX_EINVAL_SHAPE;
  if (T == 0) return VX_OK;
  if (!x || !routes || !scores || !out || !aligned16(x)) return VX_EINVAL_SHAPE;
  if (!workspace || workspace_bytes < vx_moe_experts_workspace(T, W)) return VX_EWORKSPACE;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  Carver c(workspace);
  ExpertScratch es = carve_experts(c, T, dm);
  profile_mark(st, "");
  s = run_experts(x, T, routes, W, dm, es, st);
  if (s) return s;
  cudaError_t e = launch_combine_partial(es.yd, dm.d, es.inverse, scores, T, dm.k, dm.d, out, st);
  if (e != cudaSuccess) return vx_cuda_fail(e);
  profile_mark(st, "combine_partial");
  return VX_OK;
}

size_t vx_moe_block_workspace(int32_t T, const vx_moe_weights* W) {
  if (!W || T < 0) return 0;
  const bool shared = W->shared_gate.w != nullptr;
  BlockDims dm{W->num_experts, W->hidden, W->top_k, W->gate.out, shared ? W->shared_gate.out : 0,
               shared, W->pool, W->expert_path};
  Carver c(nullptr);
  c.take<uint16_t>(int64_t(T) * dm.E);   // logits
  c.take<int32_t>(int64_t(T) * dm.k);    // inds
  c.take<uint16_t>(int64_t(T) * dm.k);   // weights
  c.take<uint16_t>(T);                   // sg
  carve_experts(c, T, dm, int(router_counters(T)));   // err + router arrival counters
  size_t bytes = c.size();
  if (T <= kDecodeMaxT) {   // the decode launch's (smaller) scratch fits in the same bytes
    Carver cd(nullptr);
    carve_decode(cd, T, dm);
    bytes = std::max(bytes, cd.size());
  }
  return bytes;
}

int vx_moe_block(const uint16_t* x, int32_t T, const vx_moe_weights* W, uint16_t* y, int32_t* inds,
                 uint16_t* weights, void* workspace, size_t workspace_bytes, void* stream) {
  int s = block_args_status(x, T, W, y);
  if (s || T == 0) return s;
  BlockDims dm;
  check_weights(W, true, &dm);
  if (!workspace || workspace_bytes < vx_moe_block_workspace(T, W)) return VX_EWORKSPACE;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (use_decode(T, dm)) {
    // decode-sized batch: the whole block in one cooperative launch
    Carver cd(workspace);
    DecodeScratch ds = carve_decode(cd, T, dm);
    cudaError_t e = cudaMemsetAsync(ds.words, 0, 4 * sizeof(int32_t), st);
    if (e != cudaSuccess) return vx_cuda_fail(e);
    profile_mark(st, "");
    const vx_moe_pool& pl = *dm.pool;
    DecodeArgs a{};
    a.x = x;
    a.router_w = W->router_w;
    a.router_bias = W->router_bias;
    a.keep_mass = W->keep_mass;
    a.keep_min = W->keep_min;
    if (dm.shared) a.seg = W->shared_expert_gate;
    a.gu_rec = static_cast<const unsigned char*>(pl.gate_up.records);
    a.gu_stride = tile_pool_bytes(1, dm.I, dm.d, 2, pl.gate_up.tile_rows, pl.gate_up.group_size);
    a.dn_rec = static_cast<const unsigned char*>(pl.down.records);
    a.dn_stride = tile_pool_bytes(1, dm.d, dm.I, 1, pl.down.tile_rows, pl.down.group_size);
    a.slot_of = pl.slot_of;
    a.slots = pl.slots;
    a.gu_rec_s = dm.shared ? static_cast<const unsigned char*>(pl.shared_gate_up.records) : nullptr;
    a.dn_rec_s = dm.shared ? static_cast<const unsigned char*>(pl.shared_down.records) : nullptr;
    a.T = T;
    a.E = dm.E;
    a.d = dm.d;
    a.k = dm.k;
    a.I = dm.I;
    a.Is = dm.shared ? dm.Is : 0;
    a.dn_mt = pl.down.tile_rows / 16;
    a.ldh = ds.ldh;
    a.logits = ds.logits;
    a.h = ds.h;
    a.sg = ds.sg;
    a.err = ds.words;
    a.sync = reinterpret_cast<uint32_t*>(ds.words + 2);
    a.y = y;
    a.inds_out = inds;
    a.w_out = weights;
    a.wait_ns = 1000ull * 1000 * 1000;   // a grid barrier gives up after 1 s
    e = launch_decode(a, st);
    if (e != cudaSuccess) return vx_cuda_fail(e);
    profile_mark(st, "decode");
    return VX_OK;
  }
  Carver c(workspace);
  uint16_t* logits = c.take<uint16_t>(int64_t(T) * dm.E);
  int32_t* inds_ws = c.take<int32_t>(int64_t(T) * dm.k);
  uint16_t* w_ws = c.take<uint16_t>(int64_t(T) * dm.k);
  uint16_t* sg = c.take<uint16_t>(T);
  const int n_counters = int(router_counters(T));
  ExpertScratch es = carve_experts(c, T, dm, n_counters);
  int32_t* counters = es.err + kErrWords;
  if (!inds) inds = inds_ws;
  if (!weights) weights = w_ws;
  // one memset clears the error words and the router's arrival counters
  cudaError_t e = cudaMemsetAsync(es.err, 0, size_t(kErrWords + n_counters) * sizeof(int32_t), st);
  if (e != cudaSuccess) return vx_cuda_fail(e);
  // A decode-sized batch (at most kPermSmall routes) is sorted by expert in
  // the router's last CTA.
  const bool fuse_perm = int64_t(T) * dm.k <= kPermSmall && dm.E <= kPermSmallMaxE;
  PermSmallArgs pa{dm.E, dm.shared ? T : 0, dm.k, item_chunk(expert_path(T, dm), dm), nullptr,
                   es.order, es.inverse, es.offsets, es.active, es.n_active, es.src_rows, es.err,
                   es.items, es.n_items};
  s = router_impl(x, T, W, dm, logits, inds, weights, dm.shared ? sg : nullptr, counters, st,
                  fuse_perm ? &pa : nullptr, true);
  if (s) return s;
  s = run_experts(x, T, inds, W, dm, es, st, true, fuse_perm);
  if (s) return s;
  e = launch_combine(es.yd, dm.d, es.inverse, weights, T, dm.k, dm.d,
                                 dm.shared ? kSharedInternal : kSharedNone, es.offsets, dm.E, sg,
                                 nullptr, nullptr, nullptr, y, st);
  if (e != cudaSuccess) return vx_cuda_fail(e);
  profile_mark(st, "combine");
  return VX_OK;
}

// ---- Expert parallelism over peer memory --------------------------------

size_t vx_ep_buffer_bytes(int32_t world, int32_t tokens_cap, int32_t hidden, int32_t top_k) {
  if (world < 1 || world > VX_EP_MAX_RANKS || tokens_cap < 1 || hidden < 1 || top_k < 1) return 0;
  return size_t(ep_layout(world, tokens_cap, hidden, top_k).bytes);
}

static int check_comm(const vx_ep_comm* c, int32_t T, EpArgs* a) {
  if (!c || c->world < 1 || c->world > VX_EP_MAX_RANKS || c->rank < 0 || c->rank >= c->world)
    return VX_EINVAL_SHAPE;
  if (c->hidden < 8 || c->hidden % 8 || c->top_k < 1 || c->top_k > 32 || c->tokens_cap < 1)
    return VX_EINVAL_SHAPE;
  if (c->num_experts < c->world || c->num_experts % c->world) return VX_EINVAL_SHAPE;
  if (T < 0 || T > c->tokens_cap) return VX_EINVAL_SHAPE;
  const EpLayout L = ep_layout(c->world, c->tokens_cap, c->hidden, c->top_k);
  for (int p = 0; p < VX_EP_MAX_RANKS; ++p) {
    a->buf[p] = p < c->world ? static_cast<unsigned char*>(c->buffers[p]) : nullptr;
    if (p < c->world && (!a->buf[p] || !aligned16(a->buf[p]))) return VX_EINVAL_SHAPE;
  }
  a->P = c->world;
  a->rank = c->rank;
  a->T = T;
  a->d = c->hidden;
  a->k = c->top_k;
  a->El = c->num_experts / c->world;
  a->err = c->err;
  a->wait_ns = c->wait_ns ? c->wait_ns : 20ull * 1000 * 1000 * 1000;
  a->off_x = L.x;
  a->off_ids = L.ids;
  a->off_w = L.w;
  a->off_back = L.back;
  return VX_OK;
}

typedef CUresult (*PfnMemGetAddressRange)(CUdeviceptr*, size_t*, CUdeviceptr);

static PfnMemGetAddressRange mem_range_fn() {
  static PfnMemGetAddressRange fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PfnMemGetAddressRange>(p);
  }
  return fn;
}

int vx_ep_ipc_handle(const void* buffer, void* handle, uint64_t* offset) {
  if (!buffer || !handle || !offset) return VX_EINVAL_SHAPE;
  PfnMemGetAddressRange range = mem_range_fn();
  if (!range) return VX_EUNSUPPORTED;
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, reinterpret_cast<CUdeviceptr>(buffer)) != CUDA_SUCCESS) return VX_EINVAL_SHAPE;
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return vx_cuda_fail(e);
  static_assert(sizeof(h) == VX_EP_IPC_HANDLE_BYTES, "IPC handle size");
  memcpy(handle, &h, sizeof(h));
  *offset = uint64_t(reinterpret_cast<uintptr_t>(buffer) - uintptr_t(base));
  return VX_OK;
}

int vx_ep_ipc_open(const void* handle, uint64_t offset, void** buffer) {
  if (!handle || !buffer) return VX_EINVAL_SHAPE;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return vx_cuda_fail(e);
  *buffer = static_cast<char*>(base) + offset;
  return VX_OK;
}

int vx_ep_ipc_close(void* buffer, uint64_t offset) {
  if (!buffer) return VX_EINVAL_SHAPE;
  cudaError_t e = cudaIpcCloseMemHandle(static_cast<char*>(buffer) - offset);
  return e == cudaSuccess ? VX_OK : vx_cuda_fail(e);
}

int vx_ep_dispatch(const vx_ep_comm* comm, const uint16_t* x, int32_t T, const int32_t* inds,
                   const uint16_t* weights, void* stream) {
  EpArgs a;
  int s = check_comm(comm, T, &a);
  if (s) return s;
  if (T == 0) return VX_OK;
  if (!x || !inds || !weights || !aligned16(x)) return VX_EINVAL_SHAPE;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  profile_mark(st, "");
  cudaError_t e = launch_ep_dispatch(a, x, inds, weights, st);
  if (e != cudaSuccess) return vx_cuda_fail(e);
  profile_mark(st, "ep_dispatch");
  return VX_OK;
}

// The shard's pipeline for the P*T received rows.  An AUTO expert path
// follows the rows that carry a slot here: T*k of them on average (the P*T*k
// received slots are spread over P ranks).
static int ep_dims(const vx_ep_comm* comm, int32_t T, const vx_moe_weights* W, BlockDims* dm) {
  int s = check_weights(W, false, dm);
  if (s) return s;
  if (dm->E * comm->world != comm->num_experts || dm->d != comm->hidden || dm->k != comm->top_k)
    return VX_EINVAL_SHAPE;
  dm->shared = false;
  dm->Is = 0;
  if (dm->path == VX_PATH_AUTO) {
    const int o = path_override();
    dm->path = o ? o : (int64_t(T) * dm->k >= 4 * int64_t(dm->E) ? VX_PATH_GEMM : VX_PATH_GEMV);
  }
  return VX_OK;
}

size_t vx_ep_experts_workspace(const vx_ep_comm* comm, int32_t T, const vx_moe_weights* W) {
  EpArgs a;
  BlockDims dm;
  if (check_comm(comm, T, &a) || ep_dims(comm, T, W, &dm)) return 0;
  Carver c(nullptr);
  carve_experts(c, T * comm->world, dm);
  return c.size();
}

int vx_ep_experts(const vx_ep_comm* comm, int32_t T, const vx_moe_weights* W, void* workspace,
                  size_t workspace_bytes, void* stream) {
  EpArgs a;
  int s = check_comm(comm, T, &a);
  if (s) return s;
  BlockDims dm;
  s = ep_dims(comm, T, W, &dm);
  if (s) return s;
  if (T == 0) return VX_OK;
  if (!workspace || workspace_bytes < vx_ep_experts_workspace(comm, T, W)) return VX_EWORKSPACE;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  profile_mark(st, "");
  const int rows = T * comm->world;
  Carver c(workspace);
  ExpertScratch es = carve_experts(c, rows, dm);
  cudaError_t e = cudaMemsetAsync(es.err, 0, kErrWords * sizeof(int32_t), st);
  if (e != cudaSuccess) return vx_cuda_fail(e);
  e = launch_ep_wait_dispatch(a, st);
  if (e != cudaSuccess) return vx_cuda_fail(e);
  profile_mark(st, "ep_wait");
  unsigned char* own = a.buf[a.rank];
  s = run_experts(reinterpret_cast<const uint16_t*>(own + a.off_x), rows,
                  reinterpret_cast<const int32_t*>(own + a.off_ids), W, dm, es, st, true);
  if (s) return s;
  e = launch_ep_send(a, es.yd, dm.d, es.inverse, st);
  if (e != cudaSuccess) return vx_cuda_fail(e);
  profile_mark(st, "ep_send");
  return VX_OK;
}

int vx_ep_combine(const vx_ep_comm* comm, int32_t T, const int32_t* inds, const uint16_t* shared,
                  const uint16_t* shared_gate, uint16_t* y, void* stream) {
  EpArgs a;
  int s = check_comm(comm, T, &a);
  if (s) return s;
  if ((shared == nullptr) != (shared_gate == nullptr)) return VX_EINVAL_SHAPE;
  if (T == 0) return VX_OK;
  if (!inds || !y) return VX_EINVAL_SHAPE;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  profile_mark(st, "");
  cudaError_t e = launch_ep_combine(a, inds, shared, shared_gate, y, st);
  if (e != cudaSuccess) return vx_cuda_fail(e);
  profile_mark(st, "ep_combine");
  return VX_OK;
}

int vx_weighted_combine(const void* outputs, int32_t dtype, int32_t n_out, const int32_t* routes,
                        const void* scores, int64_t T, int32_t k, int32_t d, void* y, int32_t* error_count,
                        void* stream) {
  if (dtype != VX_DTYPE_BF16 && dtype != VX_DTYPE_F32) return VX_EINVAL_DTYPE;
  if (T < 0 || T > 0x7FFFFFFF || k < 1 || d < 0 || n_out < 1 || (!routes && n_out != k)) return VX_EINVAL_SHAPE;
  if (T == 0 || d == 0) return VX_OK;
  if (!outputs || !scores || !y) return VX_EINVAL_SHAPE;
  cudaError_t e = launch_weighted_combine(outputs, n_out, routes, scores, T, k, d, dtype == VX_DTYPE_BF16, y,
                                          error_count, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? VX_OK : vx_cuda_fail(e);
}

int vx_rmsnorm(const uint16_t* x, const uint16_t* gain, int32_t T, int32_t d, float eps, uint16_t* y,
               void* stream) {
  if (T < 0 || d <= 0) return VX_EINVAL_SHAPE;
  if (T == 0) return VX_OK;
  if (!x || !gain || !y) return VX_EINVAL_SHAPE;
  cudaError_t e = launch_rmsnorm(x, gain, T, d, eps, y, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? VX_OK : vx_cuda_fail(e);
}

}  // extern "C"
