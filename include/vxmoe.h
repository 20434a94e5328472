/*
 * vxmoe.h - C ABI of the B200 (sm_100a) routed sparse-MoE block.
 *
 * Plain pointers, sizes and a cudaStream_t (passed as void*).  Every pointer
 * is device memory owned by the caller; the library allocates no device
 * memory.  Scratch space comes from a workspace the caller passes, except for
 * vx_moe_block_noalloc, which uses the library's own static device array of
 * VX_NOALLOC_SCRATCH_BYTES instead.  Every entry point is stream-ordered on
 * the caller's stream, performs no host synchronisation and returns a
 * vx_status code.
 *
 * bf16 values travel as uint16_t bit patterns.  Q4 weights use the MLX
 * affine layout of the reference: uint32 words along the input axis, element
 * i in bits 4*(i%8) of word i/8, bf16 scale and bias per group of 32 inputs,
 * w = scale*q + bias (models/flashnext/metal_runtime.py:1022-1027).
 *
 * Reference paths below are relative to the Veystrix-Core project.
 */
#ifndef VXMOE_H
#define VXMOE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes.  The Python layer maps them onto the exceptions the
 * reference raises: SHAPE/INDEX -> ValueError, DTYPE -> TypeError,
 * CUDA/UNSUPPORTED -> RuntimeError (metal_runtime.py:446-461, :839-895,
 * :138-142, :824-825). */
typedef enum vx_status {
  VX_OK = 0,
  VX_EINVAL_SHAPE = 1,
  VX_EINVAL_DTYPE = 2,
  VX_EINVAL_INDEX = 3,
  VX_ECUDA = 4,
  VX_ETIMEOUT = 5,
  VX_EWORKSPACE = 6,
  VX_EUNSUPPORTED = 7
} vx_status;

/* One packed Q4 projection bank: w [experts, out, in/8] uint32,
 * scales/biases [experts, out, in/group_size] bf16.  Mirrors
 * Q4G32Projection (metal_runtime.py:39-45). */
typedef struct vx_q4 {
  const uint32_t* w;
  const uint16_t* scales;
  const uint16_t* biases;
  int32_t experts;
  int32_t out;
  int32_t in;
  int32_t group_size;
} vx_q4;

/* A bank re-tiled into the resident expert pool (vx_q4_tile): the B200
 * counterpart of the reference's fixed-stride expert records
 * (slab_pack.py:1-25, expert_pool.py:1-22).  Expert e's records start at
 * e * vx_q4_tiles_bytes(1, out, in, nproj, tile_rows); inside, one record of
 * nproj * (tile_rows/16) * 1280 bytes per (row tile, 128-input chunk) holds
 * the packed words and the bf16 scales/biases in the order the decode GEMV
 * reads them.  nproj 2 interleaves a gate/up pair. */
typedef struct vx_q4_tiles {
  const void* records;
  int32_t experts;
  int32_t out;
  int32_t in;
  int32_t group_size;
  int32_t nproj;              /* 2: gate and up interleaved; 1: one projection */
  int32_t tile_rows;          /* 16 (gate/up) or 16/32 (single projection) */
} vx_q4_tiles;

/* The tiled pool of one block.  gate_up: routed gate+up (nproj 2, tile_rows
 * 16); down: routed down (nproj 1, tile_rows 32 or 16); shared_*: the shared
 * expert (records NULL when the block has none). */
typedef struct vx_moe_pool {
  vx_q4_tiles gate_up;
  vx_q4_tiles down;
  vx_q4_tiles shared_gate_up;
  vx_q4_tiles shared_down;
  /* Partial residency (models/flashnext/expert_pool.py:42, :123-159;
   * metal_runtime.py:198-228): when slot_of is not NULL, the routed records
   * (gate_up, down) hold `slots` experts' records ([slots] records, .experts
   * == slots) and routed expert e's are those of slot slot_of[e]
   * (device int32 [num_experts]).  The caller makes every expert a call
   * routes to resident before the call; an entry outside [0, slots) reads
   * slot 0 - that expert's output is undefined, its reads stay in bounds.
   * NULL (zero-initialised): expert e's records at e * stride. */
  const int32_t* slot_of;
  int32_t slots;
} vx_moe_pool;

/* Weights of one MoE block (adaptive_topk.py:54-293).  shared_* banks have
 * experts == 1; shared_gate.w == NULL means "no shared expert".  router_w is
 * the unquantised bf16 gate [num_experts, hidden] (preflight.py:70).  pool,
 * when not NULL, is the same experts re-tiled by vx_q4_tile: the routed and
 * shared passes then stream the pool (the MLX banks still give the shapes). */
typedef struct vx_moe_weights {
  vx_q4 gate;                 /* [E, I, d/8]  switch_mlp.gate_proj */
  vx_q4 up;                   /* [E, I, d/8]  switch_mlp.up_proj   */
  vx_q4 down;                 /* [E, d, I/8]  switch_mlp.down_proj */
  vx_q4 shared_gate;          /* [1, Is, d/8] shared_expert.gate_proj */
  vx_q4 shared_up;            /* [1, Is, d/8] shared_expert.up_proj   */
  vx_q4 shared_down;          /* [1, d, Is/8] shared_expert.down_proj */
  vx_q4 shared_expert_gate;   /* [1, 1, d/8]  mlp.shared_expert_gate  */
  const uint16_t* router_w;   /* bf16 [E, d]  mlp.gate */
  int32_t num_experts;
  int32_t hidden;
  int32_t top_k;
  const vx_moe_pool* pool;    /* may be NULL */
  /* Expert pipeline: VX_PATH_AUTO picks the grouped GEMV for decode-sized
   * batches and the tcgen05 grouped GEMM once the batch averages at least
   * four routed positions per expert (T*top_k >= 4*num_experts); under
   * AUTO, vx_moe_block runs a batch of at most 4 tokens over a tiled pool as
   * one cooperative launch (router to combine, VXMOE_DECODE=0 disables it).
   * VX_PATH_GEMV / VX_PATH_GEMM force the multi-kernel pipelines. */
  int32_t expert_path;
  /* bf16 [E] added to the bf16 router logits before softmax/top-k (rounded
   * to bf16 again), or NULL.  The skewed-load benchmark configuration adds
   * +2.0 to the logits of its hot experts this way. */
  const uint16_t* router_bias;
  /* Adaptive top-k (models/flashnext/adaptive_topk.py:44-51, :107-118,
   * :224-233): with 0 < keep_mass < 1 a token keeps its leading top-k slots
   * (descending probability) until their share of its top-k probability
   * mass reaches keep_mass, and at least keep_min of them (clamped to
   * 1..top_k); its other slots name its first expert with weight 0, so they
   * add no expert reads, and the weights are renormalised over the kept
   * mass.  keep_mass 0 (zero-initialised) or >= 1: every slot, the exact
   * top-k. */
  double keep_mass;
  int32_t keep_min;
} vx_moe_weights;

#define VX_PATH_AUTO 0
#define VX_PATH_GEMV 1
#define VX_PATH_GEMM 2

/* Library identification and error text. */
const char* vx_version(void);
const char* vx_strerror(int status);
/* Last CUDA error string seen by the library. */
const char* vx_last_cuda_error(void);

/* ---- Q4 arithmetic pieces -------------------------------------------- */

/* Dequantise one expert of a bank to float32 [out, in]: scale*q + bias.
 * Replaces mx.dequantize(..., mode="affine") (metal_runtime.py:770-777). */
int vx_q4_dequant(const vx_q4* bank, int32_t expert, float* out, void* stream);

/* Size in bytes of a tiled pool for `experts` experts of an [out, in] bank
 * (nproj 1 or 2, tile_rows 16 or 32); 0 for an invalid shape. */
size_t vx_q4_tiles_bytes(int32_t experts, int32_t out, int32_t in, int32_t nproj,
                         int32_t tile_rows);
/* The same for banks quantised with `group_size` inputs per scale/bias pair
 * (32, or 64: one pair per row per 64 inputs, kept as stored,
 * metal_runtime.py:770-777 with group_size=64). */
size_t vx_q4_tiles_bytes_group(int32_t experts, int32_t out, int32_t in, int32_t nproj,
                               int32_t tile_rows, int32_t group_size);
/* Re-tile bank a (and b, the up half of a gate/up pair, when nproj == 2;
 * same shape as a) into records (device, 16-byte aligned, records_bytes >=
 * vx_q4_tiles_bytes).  Out-of-range rows and groups are zero-filled.  A
 * one-time load step, the role of the reference's slab packing
 * (slab_pack.py:1-25); the decode passes then read each expert's records
 * with one bulk copy per chunk. */
int vx_q4_tile(const vx_q4* a, const vx_q4* b, int32_t nproj, int32_t tile_rows,
               void* records, size_t records_bytes, void* stream);

/* h = silu(g) * u over n bf16 values with MLX's bf16 rounding sequence
 * (metal_runtime.py:267-285; swiglu_contract.py:144-147). */
int vx_swiglu_bf16(const uint16_t* gate, const uint16_t* up, uint16_t* out,
                   int64_t n, void* stream);

/* MLX gather_qmm with transpose=True, mode="affine", bits=4:
 * out[b, m, :] = x[lhs[b]*M + m, :] . dequant(w[rhs[b]])^T, bf16 out
 * [B, M, N].  lhs may be NULL (identity).  sorted_indices is a hint only.
 * Replaces mx.gather_qmm (expert_cache.py:818-829). */
size_t vx_gather_qmm_workspace(int64_t B, int32_t M, int32_t experts, int64_t x_rows,
                               int32_t K);
int vx_gather_qmm(const uint16_t* x, int64_t x_rows, const vx_q4* w,
                  const int32_t* lhs, const int32_t* rhs, int64_t B, int32_t M,
                  int32_t sorted_indices, uint16_t* out, void* workspace,
                  size_t workspace_bytes, void* stream);

/* ---- Router ----------------------------------------------------------- */

/* softmax(precise) -> top-k -> selected scores -> renorm over bf16 logits
 * [T, E] (adaptive_topk.py:59-65, :257-262; compiled.py:60-70).  Top-k
 * order: bf16 logit descending, ties by lower expert id.  scores (raw
 * selected probabilities) and mass may be NULL. */
int vx_softmax_topk(const uint16_t* logits, int32_t T, int32_t E, int32_t k,
                    int32_t* inds, uint16_t* scores, uint16_t* weights,
                    uint16_t* mass, void* stream);

/* Full router: bf16 logits = x . router_w^T, then vx_softmax_topk.  Also
 * writes sg[t] = sigmoid(shared_expert_gate(x)) in bf16 when sg != NULL and
 * the weights carry a shared expert gate.  logits may be NULL. */
size_t vx_router_workspace(int32_t T, const vx_moe_weights* W);
int vx_router(const uint16_t* x, int32_t T, const vx_moe_weights* W,
              uint16_t* logits, int32_t* inds, uint16_t* weights, uint16_t* sg,
              void* workspace, size_t workspace_bytes, void* stream);

/* ---- Permutation ------------------------------------------------------ */

/* Stable sort of P expert ids by expert (mlx-vlm _gather_sort, called at
 * expert_cache.py:2017-2037): order[pos] = flat index at sorted position,
 * inverse[i] = sorted position of flat index i, offsets[E+1] = run starts.
 * Ids outside [0, E) are counted in *error_count (device int32, may be
 * NULL) and dropped. */
size_t vx_permute_workspace(int64_t P, int32_t E);
int vx_permute(const int32_t* ids, int64_t P, int32_t E, int32_t* order,
               int32_t* inverse, int32_t* offsets, int32_t* error_count,
               void* workspace, size_t workspace_bytes, void* stream);

/* ---- Routed experts and the whole block -------------------------------- */

/* The executor: routed experts for given routes [T, k] (int32 expert ids)
 * and scores [T, k] bf16 (MetalMoEExecutor.execute, metal_runtime.py:
 * 799-974).  With scores: out [T, d] = bf16(float(bf16(sum_s
 * float(bf16(y_s))*score_s)) + shared_y), where shared_y is shared_y[T, d],
 * or bf16(shared[T,d]*shared_gate[T]) when given as parts, or absent.
 * Without scores (NULL): out [T, k, d] holds each slot's bf16 output. */
size_t vx_moe_experts_workspace(int32_t T, const vx_moe_weights* W);
int vx_moe_experts(const uint16_t* x, int32_t T, const int32_t* routes,
                   const uint16_t* scores, const vx_moe_weights* W,
                   const uint16_t* shared_y, const uint16_t* shared,
                   const uint16_t* shared_gate, uint16_t* out, void* workspace,
                   size_t workspace_bytes, void* stream);

/* Expert-parallel share of the executor: routes [T, k] hold expert ids of
 * this bank or -1 (slot served elsewhere); out [T, d] float32 receives the
 * unrounded slot-order sum of bf16(y_s)*score_s over the present slots.  The
 * rank that owns the tokens adds the partials of all ranks in rank order and
 * rounds once, as the single-GPU combine does (metal_runtime.py:315-334).
 * Uses vx_moe_experts_workspace. */
int vx_moe_experts_partial(const uint16_t* x, int32_t T, const int32_t* routes,
                           const uint16_t* scores, const vx_moe_weights* W, float* out,
                           void* workspace, size_t workspace_bytes, void* stream);

/* The whole block, _moe_call at threshold 1.0 (adaptive_topk.py:54-293):
 * router, top-k, renorm, shared expert and its gate, routed experts and the
 * combine.  y [T, d] bf16.  inds/weights (may be NULL) receive the routing. */
size_t vx_moe_block_workspace(int32_t T, const vx_moe_weights* W);
int vx_moe_block(const uint16_t* x, int32_t T, const vx_moe_weights* W,
                 uint16_t* y, int32_t* inds, uint16_t* weights, void* workspace,
                 size_t workspace_bytes, void* stream);

/* The whole block without a workspace, for callers that cannot allocate
 * device memory (a plugin living inside another runtime's memory pool, or
 * code that must not call cudaMalloc once it is running).  No counterpart in
 * the reference.  Scratch comes from a static device array of
 * VX_NOALLOC_SCRATCH_BYTES inside the library, which every GPU that loads the
 * library keeps until the process exits.  Arguments are checked as
 * vx_moe_block checks them (same status codes; T == 0 returns VX_OK); then a
 * batch whose scratch (vx_moe_block_workspace) exceeds the array returns
 * VX_EWORKSPACE.  The first call on a device looks up the array's device
 * address (set-up, once per device, repeated only if the device's context
 * changes, e.g. after cudaDeviceReset); make that first call before any
 * stream capture.  All calls
 * share one array: calls that overlap on the GPU (other streams, other host
 * threads) race and must be serialised by the caller.  Allocates nothing. */
#define VX_NOALLOC_SCRATCH_BYTES (2u << 20)
int vx_moe_block_noalloc(const uint16_t* x, int32_t T, const vx_moe_weights* W,
                         uint16_t* y, int32_t* inds, uint16_t* weights, void* stream);

/* ---- Expert parallelism over NVLink peer memory ----------------------- */

/* The reference serves the block on one Apple GPU and has no exchange; these
 * entry points are the B200 scale-out of the same block: the routed experts
 * split into contiguous shards of num_experts/world per rank, one process per
 * GPU, every rank's exchange buffer mapped into every rank (CUDA IPC).  One
 * step, every rank with the same T <= tokens_cap tokens:
 *   vx_router (own tokens) -> vx_ep_dispatch -> vx_ep_experts (the rank's
 *   shard) -> [shared expert, own tokens] -> vx_ep_combine
 * Dispatch stores each token's row once into every rank that owns one of its
 * experts (peer stores over NVLink) with slot ids local to that rank; the
 * experts call waits for every rank's dispatch, runs the grouped pipeline and
 * stores each row's float32 partial sum straight into its home rank; the
 * combine waits for every rank's partials and adds them in rank order,
 * rounds once and adds bf16(shared_gate * shared), the float32-then-bf16
 * contract of the single-GPU combine (metal_runtime.py:315-334).
 * Waits are bounded: one that runs out sets a bit of *err and returns.
 * Nothing synchronises the host, so the step captures into a CUDA graph. */
#define VX_EP_MAX_RANKS 8
#define VX_EP_IPC_HANDLE_BYTES 64

typedef struct vx_ep_comm {
  void* buffers[VX_EP_MAX_RANKS]; /* every rank's exchange buffer as mapped here, own at [rank] */
  int32_t rank, world;
  int32_t tokens_cap;             /* tokens per rank and step, at most */
  int32_t hidden, top_k;
  int32_t num_experts;            /* routed experts over all ranks */
  int32_t* err;                   /* device word or NULL: bit 0 dispatch wait ran out, bit 1 combine */
  uint64_t wait_ns;               /* bound of every wait in ns (0: 20 s) */
} vx_ep_comm;

/* Bytes of one rank's exchange buffer.  The caller allocates it on its GPU,
 * zeroes it, and lets no rank dispatch before every rank has zeroed its own
 * (a host barrier); one buffer serves any number of layers run in the same
 * order on every rank. */
size_t vx_ep_buffer_bytes(int32_t world, int32_t tokens_cap, int32_t hidden, int32_t top_k);

/* CUDA IPC of an exchange buffer: handle (VX_EP_IPC_HANDLE_BYTES) and offset
 * of `buffer` inside its allocation; a peer process opens them into its own
 * mapping and closes that mapping when done. */
int vx_ep_ipc_handle(const void* buffer, void* handle, uint64_t* offset);
int vx_ep_ipc_open(const void* handle, uint64_t offset, void** buffer);
int vx_ep_ipc_close(void* buffer, uint64_t offset);

/* inds/weights [T, k]: the router's global expert ids and slot weights. */
int vx_ep_dispatch(const vx_ep_comm* comm, const uint16_t* x, int32_t T, const int32_t* inds,
                   const uint16_t* weights, void* stream);

/* W: this rank's shard (num_experts/world routed experts, no shared expert). */
size_t vx_ep_experts_workspace(const vx_ep_comm* comm, int32_t T, const vx_moe_weights* W);
int vx_ep_experts(const vx_ep_comm* comm, int32_t T, const vx_moe_weights* W, void* workspace,
                  size_t workspace_bytes, void* stream);

/* y [T, d] bf16 for this rank's tokens; shared [T, d] and shared_gate [T]
 * bf16, both or neither. */
int vx_ep_combine(const vx_ep_comm* comm, int32_t T, const int32_t* inds, const uint16_t* shared,
                  const uint16_t* shared_gate, uint16_t* y, void* stream);

/* Combine of already projected values, the reference's generic helper
 * weighted_combine (metal_runtime.py:145-191): y[t, :] = sum_s out[t, sel, :]
 * * scores[t, s] with sel = routes[t, s] when the outputs hold all n_out
 * experts of a token (out [T, n_out, d]), else sel = s (routes NULL, out
 * [T, k, d], n_out == k).  dtype VX_DTYPE_BF16 or VX_DTYPE_F32 for outputs,
 * scores and y alike; bf16 products are rounded to bf16, the slot sum runs in
 * float32 in slot order and is rounded once.  Routes outside [0, n_out) add
 * nothing and are counted in *error_count (device int32, may be NULL). */
#define VX_DTYPE_BF16 0
#define VX_DTYPE_F32 1
int vx_weighted_combine(const void* outputs, int32_t dtype, int32_t n_out, const int32_t* routes,
                        const void* scores, int64_t T, int32_t k, int32_t d, void* y,
                        int32_t* error_count, void* stream);

/* RMSNorm in float32 with a bf16 gain, bf16 out (patch_rmsnorm.py:96-120). */
int vx_rmsnorm(const uint16_t* x, const uint16_t* gain, int32_t T, int32_t d,
               float eps, uint16_t* y, void* stream);

/* ---- Stage timing ----------------------------------------------------- */

/* Per-kernel boundary timing, the role of the reference's BoundaryProfiler
 * (boundary_profiler.py:1-25; used at metal_runtime.py:618-637).  While
 * enabled, vx_moe_block / vx_moe_experts / vx_router record a CUDA event on
 * the caller's stream after each kernel.  Enabling resets the records.
 * vx_profile_read waits for the last event and returns, per stage label,
 * the number of launches and their average duration in milliseconds;
 * labels are written newline-separated into `labels`. */
int vx_profile_enable(int enabled);
int vx_profile_read(int max_stages, char* labels, int labels_cap, double* avg_ms,
                    int32_t* counts, int32_t* n_stages);

#ifdef __cplusplus
}
#endif

#endif /* VXMOE_H */
