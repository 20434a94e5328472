// Host-side launchers shared between the kernel files and the C ABI layer.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "vxmoe.h"

namespace vx {

// Whether chained launches carry the programmatic-serialisation attribute:
// VXMOE_PDL=0 never, 1 every chained launch, 2 (default) only the short
// glue kernels (router, permutation, records, combine, exchange) - the
// streaming GEMV/GEMM kernels launch plainly.  The kernels are correct
// either way.
bool chain_enabled(bool streaming);

// Launches `kernel` with programmatic stream serialisation, so that the
// grid may be scheduled while the previous kernel on the stream finishes;
// the kernel must call chain_begin() or chain_wait() before its first
// global-memory access.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_chained_as(bool streaming, void (*kernel)(KArgs...), dim3 grid, dim3 block,
                                     size_t smem, cudaStream_t st, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = chain_enabled(streaming) ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

template <typename... KArgs, typename... Args>
inline cudaError_t launch_chained(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                                  cudaStream_t st, Args... args) {
  return launch_chained_as(false, kernel, grid, block, smem, st, args...);
}

template <typename... KArgs, typename... Args>
inline cudaError_t launch_streaming(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                                    cudaStream_t st, Args... args) {
  return launch_chained_as(true, kernel, grid, block, smem, st, args...);
}

// Tokens per work item of the tensor-pipe GEMV (an expert's run is cut into
// items of at most this many positions).  The GEMV's block-diagonal B holds
// two tokens per MMA.
constexpr int kItemChunk = 2;

struct MmaArgs {
  CUtensorMap tm_b0, tm_b1;  // 2-D views of the packed words (set by the launcher)
  CUtensorMap tm_s0, tm_s1;
  int32_t* err;              // bit 8 set when a pipeline wait ran out (may be null)
  vx_q4 b0, b1;              // routed banks (b1: up in gate/up mode)
  vx_q4 s0, s1;              // shared expert banks (expert id E)
  int E;
  const int32_t* items;      // [n][3] expert, first position, count
  const int32_t* n_items;
  const int32_t* src_rows;   // x row of each position (null: identity)
  const int32_t* dst_rows;   // out row of each position (null: identity)
  const uint16_t* x;         // activations in B order (see b_order_col)
  int64_t ldx;
  const float* xsum;         // [rows][ldxs] sum(x) per group, or null: sum on the tensor pipe
  int64_t ldxs;
  uint16_t* out;             // gate/up mode writes B order, projection mode plain rows
  int64_t ldo;
  int tiles_per_item;        // set by the launcher
};

// x [rows, K] bf16 -> xb [rows, K] in B order and xs [rows, ldxs] float32
// per-group sums (ldxs = K/32 rounded up to even; the pad column is zero).
cudaError_t launch_xprep(const uint16_t* x, int64_t rows, int K, uint16_t* xb, float* xs,
                         int64_t ldxs, cudaStream_t st);
inline int64_t xsum_stride(int K) { return ((K / 32) + 1) & ~1; }

cudaError_t launch_gemv_mma(bool gateup, const MmaArgs& a, int max_items, int max_out,
                            cudaStream_t st);

// Tiled expert pool: bytes of one record per (projection, 16-row m-tile) and
// 128-input chunk: 1024 of packed words + 256 of scales and biases.
constexpr int kTileRecordUnit = 1280;
// Bytes of one (projection, 16-row tile, 128-input chunk) record unit: 1,024
// of packed words, then the scale/bias pairs - 256 bytes for groups of 32,
// 128 for native groups of 64 (one pair per row and 64 inputs).
__host__ __device__ constexpr int tile_unit_bytes(int group) { return group == 64 ? 1152 : kTileRecordUnit; }

// Tokens per work item of the tiled GEMV: two B operands of two tokens each
// share every unpacked weight fragment.
constexpr int kTiledItemChunk = 4;

// Activation records of the tiled GEMV: per (128-input chunk, position) 320
// bytes - the chunk's 128 inputs in lane order [i][c] (8 inputs each, B
// order inside), then the four group sums as float32 and the record's
// inverse scale, then padding.  An item's positions are consecutive, so one
// bulk copy brings all its tokens.  The 320-byte pitch puts the two tokens a
// B operand reads on disjoint banks.
constexpr int kActRecord = 320;
constexpr int kActXsum = 256;
// act_records_kernel writes f16 records (every record of a position scaled
// by the same power of two) of x (gate/up's input) and of h (down's input,
// from the plain h rows the gate/up pass writes); both GEMV passes read them
// with the f16 unpack.
constexpr bool kActF16 = true;

struct TiledArgs {
  int32_t* err;                 // bit 8 set when a pipeline wait ran out (may be null)
  const unsigned char* rec_b;   // routed experts' records
  int64_t stride_b;             // bytes per routed expert
  const unsigned char* rec_s;   // shared expert's records (expert id E), may be null
  int N_b, N_s;                 // output rows of the routed / shared projection
  int K_b, K_s;                 // inputs of the routed / shared projection
  int E;
  const int32_t* items;         // [n][3] expert, first position, count (<= kTiledItemChunk)
  const int32_t* n_items;
  const unsigned char* act;     // activation records [chunk][act_rows][kActRecord]
  int64_t act_rows;             // positions per chunk of act
  uint16_t* out;                // plain rows [position][ldo]: h (gate/up) or the projection
  int64_t ldo;
  int tiles_per_item;           // set by the launcher
  const int32_t* slot_of;       // partial residency: routed expert -> record slot (may be null)
  int slots;
  int32_t* task_ctr;            // zero at launch: tasks after the first wave are taken from it
                                // (null: a static round robin)
};

// x rows (token src_rows[p] for position p < *n_rows, or p when src_rows is
// null) -> activation records with group sums; chunk padding is zero.
cudaError_t launch_act_records(const uint16_t* x, int64_t ldx, int K, const int32_t* src_rows,
                               const int32_t* n_rows, int64_t rows, unsigned char* act,
                               cudaStream_t st);
inline int64_t act_record_bytes(int K, int64_t rows) {
  return int64_t((K + 127) / 128) * rows * kActRecord;
}

// Grouped expert GEMM on tcgen05 (prefill).  Items of up to kGemmItemChunk
// positions; B operand rows in B order ([rows][ld] bf16).
constexpr int kGemmItemChunk = 128;

struct GemmArgs {
  CUtensorMap tm[2][4];      // [routed, shared][box rows 16, 32, 64, 128] (set by the launcher)
  int32_t* err;              // bit 9 set when a pipeline wait ran out (may be null)
  vx_q4 b0, b1;              // routed banks (b1: up in gate/up mode)
  vx_q4 s0, s1;              // shared expert banks (expert id E)
  int E;
  const int32_t* items;      // [n][3] expert, first position, count (<= kGemmItemChunk)
  const int32_t* n_items;
  uint16_t* out;             // gate/up: h rows in B order; projection: plain rows
  int64_t ldo;
  int row_tiles;             // set by the launcher
};

cudaError_t launch_gemm_tc(bool gateup, GemmArgs a, const uint16_t* x, int64_t rows, int64_t ldx,
                           int max_items, cudaStream_t st);

// bf16 rows [rows][ld] as a 2-D tensor [rows][K] (columns >= K read as zero),
// box 64 columns (128 bytes, 128-byte swizzle) x box_rows rows.
cudaError_t encode_rows(CUtensorMap* m, const uint16_t* p, int64_t rows, int K, int64_t ld, int box_rows);

// The persistent tcgen05 GEMM over the tiled pool: items of up to
// kPoolGemmItemChunk positions, weights and scales from the pool's records.
constexpr int kPoolGemmItemChunk = 64;

struct PoolGemmArgs {
  CUtensorMap tm[2][3];         // [routed, shared][box rows 16, 32, 64] (set by the launcher)
  int32_t* err;                 // bit 9 set when a pipeline wait ran out (may be null)
  const unsigned char* rec_b;   // routed records, stride_b bytes per expert
  int64_t stride_b;
  const unsigned char* rec_s;   // shared records (expert id E), may be null
  int N_b, N_s, K_b, K_s;       // outputs and inputs, routed / shared
  int tile_rows;                // rows per record (16 or 32)
  int E;
  const int32_t* items;         // [n][3] expert, first position, count (<= kPoolGemmItemChunk)
  const int32_t* n_items;
  uint16_t* out;                // gate/up: h rows in B order; projection: plain rows
  int64_t ldo;
  int row_tiles;                // 128-row tiles per item (set by the launcher)
  int max_tasks;                // upper bound of item x row-tile tasks (set by the launcher)
  const int32_t* slot_of;       // partial residency: routed expert -> record slot (may be null)
  int slots;
  int group;                    // records' quant group: 32 or 64 (native G64 pairs)
};

cudaError_t launch_gemm_pool(bool gateup, PoolGemmArgs a, const uint16_t* x, int64_t rows, int64_t ldx,
                             int max_items, cudaStream_t st);
cudaError_t launch_gather_border(const uint16_t* x, int64_t ldx, int K, const int32_t* src_rows,
                                 const int32_t* n_rows, int64_t rows, uint16_t* out, cudaStream_t st);

int64_t tile_pool_bytes(int64_t experts, int out, int in, int nproj, int tile_rows, int group = 32);
cudaError_t launch_tile_pack(const vx_q4& a, const vx_q4& b, int nproj, int tile_rows, void* out,
                             cudaStream_t st, int group = 32);
cudaError_t launch_gemv_tiled(bool gateup, int tile_rows, const TiledArgs& a, int max_items,
                              int max_out, cudaStream_t st, int group = 32);

// Upper bound of the number of work items for P routed positions over E
// experts plus Ts shared-expert positions.
inline int max_items_bound(int64_t P, int E, int Ts) {
  int64_t routed = (P + kItemChunk - 1) / kItemChunk + (P < E ? P : E);
  if (routed > P) routed = P;
  return int(routed + (Ts + kItemChunk - 1) / kItemChunk);
}

int sm_count();

// Stable sort by expert.  blk: scratch of permute_scratch_ints(P, E) ints
// (null or zero-sized: the one-CTA variant regardless of P).
cudaError_t launch_permute(const int32_t* ids, int64_t P, int E, int shared_items, int k_div,
                           const int32_t* src_map, int32_t* order, int32_t* inverse,
                           int32_t* offsets, int32_t* active, int32_t* n_active,
                           int32_t* src_rows, int32_t* err, int item_chunk, int32_t* items,
                           int32_t* n_items, int32_t* blk, cudaStream_t st);
int64_t permute_scratch_ints(int64_t P, int E);

// Decode-sized permutations (at most kPermSmall ids, E <= kPermSmallMaxE) run
// in one 256-thread CTA: the one-CTA permute kernel, or the fused router's
// last CTA when it is handed these outputs (PermSmallArgs::order non-null).
constexpr int kPermSmall = 1024;
constexpr int kPermSmallMaxE = 1024;

struct PermSmallArgs {
  int E, shared_items, k_div, item_chunk;
  const int32_t* src_map;
  int32_t *order, *inverse, *offsets, *active, *n_active, *src_rows, *err, *items, *n_items;
};

cudaError_t launch_router_logits(const uint16_t* x, int T, const uint16_t* wg, int E, int K,
                                 uint16_t* logits, cudaStream_t st);
cudaError_t launch_shared_gate(const uint16_t* x, int T, const vx_q4& seg, uint16_t* sg,
                               cudaStream_t st);
cudaError_t launch_softmax_topk(const uint16_t* logits, int T, int E, int k, int32_t* inds,
                                uint16_t* scores, uint16_t* weights, uint16_t* mass,
                                cudaStream_t st, double keep_mass = 0.0, int keep_min = 1);
// Logits, top-k/renorm, (seg != null) the shared-expert gate and (perm !=
// null; T*k <= kPermSmall) the expert sort of the routes in one launch;
// bias (bf16 [E] or null) is added to the bf16 logits; counters:
// router_counters(T) ints of scratch, zeroed by the launcher unless the
// caller cleared them earlier on the stream (counters_zeroed).
inline int64_t router_counters(int64_t T) { return (T + 7) / 8 + 1; }
struct PermSmallArgs;
// Prefill-sized batches (T >= kRouterTiledMinT, K <= 2048): logits by
// 64 x 64 tiles staged in shared memory (the same bits as the fused kernel),
// then the softmax/top-k kernel and the shared-expert gate kernel.  No
// counters, no permutation.
constexpr int kRouterTiledMinT = 256;
bool router_tiled_fits(int T, int K);
cudaError_t launch_router_tiled(const uint16_t* x, int T, const uint16_t* wg, int E, int K, int k,
                                const vx_q4* seg, uint16_t* logits, int32_t* inds, uint16_t* weights,
                                uint16_t* sg, const uint16_t* bias, cudaStream_t st, double keep_mass = 0.0,
                                int keep_min = 1);
cudaError_t launch_router_fused(const uint16_t* x, int T, const uint16_t* wg, int E, int K, int k,
                                const vx_q4* seg, uint16_t* logits, int32_t* inds, uint16_t* weights,
                                uint16_t* sg, int32_t* counters, const PermSmallArgs* perm,
                                const uint16_t* bias, cudaStream_t st, bool counters_zeroed = false,
                                double keep_mass = 0.0, int keep_min = 1);

// The whole block for at most kDecodeMaxT tokens in one cooperative launch
// (vx_decode.cu): weights from the tiled pool (gate/up records of 16 rows,
// down records of 16 or 32 rows).  Scratch (caller workspace): logits
// [T][E], sg [T], the SwiGLU outputs h [T*k+T][ldh] bf16 of every sorted
// position, and the two barrier counters in sync[2], zero at launch.
constexpr int kDecodeMaxT = 4;

struct DecodeArgs {
  const uint16_t* x;
  const uint16_t* router_w;
  const uint16_t* router_bias;        // may be null
  vx_q4 seg;                          // shared expert gate (w null: none)
  const unsigned char* gu_rec;        // routed gate/up records
  const unsigned char* gu_rec_s;      // shared gate/up records (null: no shared expert)
  const unsigned char* dn_rec;        // routed down records
  const unsigned char* dn_rec_s;      // shared down records
  int64_t gu_stride, dn_stride;       // bytes per routed expert
  int T, E, d, k, I, Is, dn_mt, ldh;  // Is = 0: no shared expert; dn_mt = down tile rows / 16
  uint16_t* logits;
  uint16_t* h;
  uint16_t* sg;
  uint32_t* sync;
  int32_t* err;                       // [0] bits 0x400 (a grid barrier wait ran out), 0x100 (a copy
                                      // wait); [1] routes dropped for an id outside [0, E)
  uint16_t* y;
  int32_t* inds_out;                  // may be null
  uint16_t* w_out;                    // may be null
  uint64_t wait_ns;
  int smem_bytes;                     // set by the launcher
  double keep_mass;                   // adaptive top-k (vx_moe_weights.keep_mass)
  int keep_min;
  const int32_t* slot_of;             // partial residency: routed expert -> record slot (may be null)
  int slots;
};

bool decode_supported(int T, int E, int d, int k, int I, int Is, int gu_tile_rows, int dn_tile_rows);
cudaError_t launch_decode(const DecodeArgs& a, cudaStream_t st);

// Expert-parallel exchange buffer of one rank (vx_ep.cu): a 256-byte header
// (u32 flag_dispatch[8], flag_combine[8], epoch, tickets[3]), then, for a step
// of T <= cap tokens per rank, rows i = r*T + t of
//   x    [P*T][d] bf16    rows received from rank r for this rank's experts
//   ids  [P*T][k] int32   their slot ids local to this rank (-1: elsewhere)
//   w    [P*T][k] bf16    their slot weights
//   back [P*T][d] float32 partial sums of this rank's tokens from rank r
// (each region sized for cap, 256-byte aligned).
constexpr int kEpMaxRanks = 8;
constexpr int64_t kEpHeaderBytes = 256;

struct EpLayout {
  int64_t x, ids, w, back, bytes;
};
EpLayout ep_layout(int P, int cap, int d, int k);

struct EpArgs {
  unsigned char* buf[kEpMaxRanks];   // every rank's exchange buffer (own at [rank])
  int P, rank, T, d, k, El;          // El: experts per rank
  int32_t* err;                      // bit 0: dispatch wait ran out, bit 1: combine wait (may be null)
  uint64_t wait_ns;                  // bound of every wait
  int64_t off_x, off_ids, off_w, off_back;
};

cudaError_t launch_ep_dispatch(const EpArgs& a, const uint16_t* x, const int32_t* inds,
                               const uint16_t* wts, cudaStream_t st);
cudaError_t launch_ep_wait_dispatch(const EpArgs& a, cudaStream_t st);
cudaError_t launch_ep_send(const EpArgs& a, const uint16_t* yd, int64_t ldy, const int32_t* inverse,
                           cudaStream_t st);
cudaError_t launch_ep_combine(const EpArgs& a, const int32_t* inds, const uint16_t* shared,
                              const uint16_t* sg, uint16_t* y, cudaStream_t st);

// Combine modes for the shared part.
enum SharedMode { kSharedNone = 0, kSharedInternal = 1, kSharedY = 2, kSharedParts = 3 };

cudaError_t launch_combine(const uint16_t* yd, int64_t ldy, const int32_t* inverse,
                           const uint16_t* weights, int T, int k, int d, SharedMode mode,
                           const int32_t* offsets, int E, const uint16_t* sg,
                           const uint16_t* shared_y, const uint16_t* shared,
                           const uint16_t* shared_gate, uint16_t* y, cudaStream_t st);
cudaError_t launch_combine_partial(const uint16_t* yd, int64_t ldy, const int32_t* inverse,
                                   const uint16_t* weights, int T, int k, int d, float* out,
                                   cudaStream_t st);
cudaError_t launch_unpermute(const uint16_t* yd, int64_t ldy, const int32_t* inverse, int T,
                             int k, int d, uint16_t* out, cudaStream_t st);
cudaError_t launch_weighted_combine(const void* outputs, int n_out, const int32_t* routes, const void* scores,
                                    int64_t T, int k, int d, bool bf16, void* y, int32_t* err,
                                    cudaStream_t st);
cudaError_t launch_rmsnorm(const uint16_t* x, const uint16_t* gain, int T, int d, float eps,
                           uint16_t* y, cudaStream_t st);
cudaError_t launch_swiglu(const uint16_t* g, const uint16_t* u, uint16_t* out, int64_t n,
                          cudaStream_t st);
cudaError_t launch_dequant(const vx_q4& bank, int expert, float* out, cudaStream_t st);
cudaError_t launch_gather_items(const int32_t* lhs, const int32_t* rhs, int64_t B, int M,
                                int64_t x_rows, int32_t* keys, int32_t* src_map, cudaStream_t st);

}  // namespace vx
