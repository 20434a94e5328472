"""CPU oracle for the routed sparse-MoE block (TEST INFRASTRUCTURE ONLY).

This module is the checker, never the product.  Only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` leg of ``bench.py`` may
import it.  The CUDA library under ``veystrix-core_b200`` never calls it and
has no CPU fallback.

It restates, in NumPy, the arithmetic of the reference block
(``models/flashnext`` of Veystrix-Core, paths below relative to that
project):

* Q4 nibble order and affine dequant: ``metal_runtime.py:1022-1027``
  (element ``i`` of a row lives in bits ``4*(i%8)`` of word ``i//8``;
  ``w = scale*q + bias``).
* Q4 matrix-vector product (MLX ``qmv``): per group ``scale*sum(x*q) +
  bias*sum(x)`` with float accumulation (``metal_runtime.py:1014-1029``; the
  same formula the Metal helpers use, ``metal_runtime.py:352-424``).
* Router: ``softmax(precise=True)`` over the bf16 gate logits, top-k,
  selected scores and their mass (``adaptive_topk.py:59-65``,
  ``compiled.py:60-64``); renormalisation ``scores / mass`` at blend 1.0
  (``adaptive_topk.py:257-262``); adaptive top-k below threshold 1.0: the
  keep rule ``_keep_for_mass`` and the dropped slots' masking
  (``adaptive_topk.py:44-51``, ``:107-118``, ``:224-233``).
* SwiGLU as MLX's bf16 sequence: ``t=exp(|g|)``, ``s=1/(1+t)``,
  ``sigma = g<0 ? s : 1-s``, ``silu=g*sigma``, ``h=silu*u``, every step
  rounded to bf16 (``metal_runtime.py:267-285``;
  ``tests/bench/swiglu_contract.py:144-147`` and ``:210-218``).
* Shared expert and its sigmoid gate (``adaptive_topk.py:264-265``).
* Fused down + score combine: each slot's down result is rounded to bf16,
  multiplied by its score and accumulated in float32 in slot order, then
  ``+ shared_y`` and a cast to bf16 (``metal_runtime.py:291-336``,
  ``:404-410``).
* The generic combine ``(y*scores).sum(-2) + shared_gate*shared``
  (``adaptive_topk.py:275-278``; ``metal_runtime.py:145-191``).
* Sort-by-expert permutation of mlx-vlm ``_gather_sort``/``_scatter_unsort``
  (called at ``expert_cache.py:2017-2037``): a stable argsort of the flat
  expert ids and its inverse.
* RMSNorm in float32 with a gain (``patch_rmsnorm.py:96-120``).

Pinning.  The Q4 unpack, the dequantised weights, the ``qmv`` formula, the
executor's float32 reference path and ``weighted_combine`` are pinned
against the reference's own NumPy code (``tests/golden``).  The bf16 router
softmax, the top-k tie order and the bf16 SwiGLU sequence live in MLX, which
is absent here; for those the restatement defines parity ("parity unpinned"
by reference data).

Top-k tie rule.  MLX's ``argpartition`` leaves the order of ties open.  The
oracle ranks experts by their bf16 logit (descending), then by expert index
(ascending).  Softmax is monotone, so the chosen set is always a valid top-k
of the probabilities, and it does not depend on how ``exp`` rounds.
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import Sequence

import numpy as np

GROUP_SIZE = 32
BITS = 4


# --------------------------------------------------------------------------
# bf16 helpers (values are carried as float32 arrays holding bf16 values)
# --------------------------------------------------------------------------


def bf16_round(a) -> np.ndarray:
    """Round float32 values to the nearest bf16 (ties to even)."""
    a = np.ascontiguousarray(np.asarray(a, dtype=np.float32))
    bits = a.view(np.uint32).astype(np.uint64)
    lsb = (bits >> 16) & 1
    rounded = ((bits + 0x7FFF + lsb) & 0xFFFF0000).astype(np.uint32)
    out = rounded.view(np.float32).copy()
    nan = np.isnan(a)
    if nan.any():
        out[nan] = np.float32("nan")
    return out.reshape(a.shape)


def bf16_bits(a) -> np.ndarray:
    """bf16 encodings (uint16) of values that are already bf16."""
    a = np.ascontiguousarray(bf16_round(a))
    return (a.view(np.uint32) >> 16).astype(np.uint16)


def bf16_from_bits(bits) -> np.ndarray:
    """float32 values of uint16 bf16 encodings."""
    bits = np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16
    return bits.view(np.float32)


def f32(a) -> np.ndarray:
    return np.asarray(a, dtype=np.float32)


# --------------------------------------------------------------------------
# Q4 affine group-32 weights
# --------------------------------------------------------------------------


def q4_unpack(w) -> np.ndarray:
    """Codes of packed uint32 words: element i = (w[i//8] >> 4*(i%8)) & 15.

    Follows ``metal_runtime.py:1022``.
    """
    w = np.asarray(w)
    if w.dtype != np.uint32:
        raise TypeError("Q4 weights must use uint32 packed values")
    shifts = (4 * np.arange(8, dtype=np.uint32))
    q = (w[..., :, None] >> shifts) & np.uint32(15)
    return q.reshape(*w.shape[:-1], w.shape[-1] * 8).astype(np.uint8)


def q4_pack(q) -> np.ndarray:
    """Inverse of :func:`q4_unpack` (codes 0..15, last axis a multiple of 8)."""
    q = np.asarray(q).astype(np.uint32)
    if q.shape[-1] % 8:
        raise ValueError("last axis must be a multiple of 8")
    q = q.reshape(*q.shape[:-1], q.shape[-1] // 8, 8)
    shifts = (4 * np.arange(8, dtype=np.uint32))
    return np.bitwise_or.reduce(q << shifts, axis=-1).astype(np.uint32)


def dequantize(w, scales, biases, group_size: int = GROUP_SIZE) -> np.ndarray:
    """float32 ``scale*q + bias`` per group (``metal_runtime.py:1026-1027``).

    ``scale*q`` is exact in float32 (8-bit by 4-bit significands), so this
    is one rounding of the exact affine value; a fused multiply-add gives
    the same bits.
    """
    q = q4_unpack(w).astype(np.float64)
    s = np.repeat(f32(scales).astype(np.float64), group_size, axis=-1)
    b = np.repeat(f32(biases).astype(np.float64), group_size, axis=-1)
    return (s * q + b).astype(np.float32)


def qmv(x, w, scales, biases, group_size: int = GROUP_SIZE) -> np.ndarray:
    """``x @ dequant(w).T`` by the MLX qmv formula, float64 accumulation.

    ``x``: [..., K] (bf16 values); ``w``: [N, K/8] uint32; scales/biases
    [N, K/group].  Returns float64 [..., N] before any output rounding:
    ``sum_g scale[n,g]*sum_i x_i q_i + bias[n,g]*sum_i x_i``.
    """
    x = np.asarray(x, dtype=np.float64)
    K = x.shape[-1]
    N = w.shape[0]
    if w.shape[-1] * 8 != K:
        raise ValueError(f"weight shape {w.shape} does not match input width {K}")
    G = K // group_size
    q = q4_unpack(w).astype(np.float64).reshape(N, G, group_size)
    xg = x.reshape(*x.shape[:-1], G, group_size)
    qsum = np.einsum("...gi,ngi->...ng", xg, q)
    xsum = xg.sum(axis=-1)[..., None, :]
    s = f32(scales).astype(np.float64)
    b = f32(biases).astype(np.float64)
    return (qsum * s + xsum * b).sum(axis=-1)


def numpy_projection(x, routes, w, scales, biases, output_width, slot_input,
                     group_size: int = GROUP_SIZE) -> np.ndarray:
    """Vectorised twin of the reference's ``_numpy_projection``.

    ``metal_runtime.py:997-1029``: float64 accumulation per output, one
    cast to ``x.dtype`` at the end.
    """
    x = np.asarray(x)
    routes = np.asarray(routes)
    tokens, slots = routes.shape
    out = np.zeros((tokens, slots, output_width), dtype=np.float64)
    for token in range(tokens):
        for slot in range(slots):
            e = int(routes[token, slot])
            src = x[token, slot] if slot_input else x[token]
            out[token, slot] = qmv(src, w[e], scales[e], biases[e], group_size)
    return out.astype(x.dtype)


# --------------------------------------------------------------------------
# bf16 elementwise contracts
# --------------------------------------------------------------------------


def _bf16_exp(v) -> np.ndarray:
    """bf16 of a float32 exp: MLX evaluates bf16 exp as float exp, then
    rounds.  float64 exp rounded to float32 stands for a correctly rounded
    float32 exp."""
    return bf16_round(np.exp(np.asarray(v, dtype=np.float64)).astype(np.float32))


def sigmoid_bf16(z) -> np.ndarray:
    """MLX's stable bf16 sigmoid: every operation rounded to bf16.

    ``metal_runtime.py:275-281``: ``t=exp(|z|)``, ``s=1/(1+t)``,
    ``sigma = z<0 ? s : 1-s``.
    """
    z = bf16_round(z)
    t = _bf16_exp(np.abs(z))
    den = bf16_round(np.float32(1) + t)
    with np.errstate(divide="ignore"):
        small = bf16_round(np.float32(1) / den)
    return np.where(z < 0, small, bf16_round(np.float32(1) - small)).astype(np.float32)


def silu_mul_bf16(gate, up) -> np.ndarray:
    """``h = silu(g) * u`` as MLX computes it in bf16.

    ``swiglu_contract.py:144-147`` (``nn.silu(gate) * up`` in bf16) with the
    sigmoid sequence of ``metal_runtime.py:267-285``.
    """
    g = bf16_round(gate)
    u = bf16_round(up)
    sig = sigmoid_bf16(g)
    silu = bf16_round(g * sig)
    return bf16_round(silu * u)


# --------------------------------------------------------------------------
# Router
# --------------------------------------------------------------------------


def router_logits(x, wg) -> np.ndarray:
    """bf16 logits of the unquantised bf16 gate (``adaptive_topk.py:60``)."""
    acc = np.asarray(x, dtype=np.float64) @ f32(wg).astype(np.float64).T
    return bf16_round(acc.astype(np.float32))


def softmax_bf16(logits) -> np.ndarray:
    """``softmax(precise=True)`` of bf16 logits: float32 math, bf16 out.

    ``p = exp(l - max) * (1 / sum)``.
    """
    l = f32(logits)
    m = l.max(axis=-1, keepdims=True)
    e = np.exp((l - m).astype(np.float64)).astype(np.float32)
    s = e.sum(axis=-1, dtype=np.float32, keepdims=True)
    inv = (np.float32(1) / s).astype(np.float32)
    return bf16_round(e * inv)


def topk_order(logits, k: int) -> np.ndarray:
    """Top-k expert ids per row: bf16 logit descending, then index ascending."""
    l = f32(logits)
    n = l.shape[-1]
    flat = l.reshape(-1, n)
    out = np.empty((flat.shape[0], k), dtype=np.int32)
    idx = np.arange(n)
    for r in range(flat.shape[0]):
        # lexsort: last key is primary
        order = np.lexsort((idx, -flat[r].astype(np.float64)))
        out[r] = order[:k]
    return out.reshape(*l.shape[:-1], k)


@dataclass
class RouterOut:
    logits: np.ndarray      # bf16 [.., E]
    probs: np.ndarray       # bf16 [.., E]
    inds: np.ndarray        # int32 [.., k]
    scores: np.ndarray      # bf16 [.., k] selected probabilities
    mass: np.ndarray        # bf16 [.., 1]
    weights: np.ndarray     # bf16 [.., k] renormalised scores


def renorm(scores, mass, blend: float = 1.0) -> np.ndarray:
    """``scores / (mass + blend*(sum(scores) - mass))`` in bf16
    (``adaptive_topk.py:257-262``)."""
    scores = f32(scores)
    sel = bf16_round(scores.sum(axis=-1, keepdims=True, dtype=np.float32))
    diff = bf16_round(sel - f32(mass))
    norm = bf16_round(f32(mass) + bf16_round(np.float32(blend) * diff))
    return bf16_round(scores / norm)


def keep_for_mass(weights, threshold: float) -> int:
    """``_keep_for_mass`` (``adaptive_topk.py:44-51``): the number of leading
    weights whose running share of their sum first reaches ``threshold``,
    in Python floats, left to right; all of them when none does."""
    total = sum(float(w) for w in weights)
    accumulated = 0.0
    for position, weight in enumerate(weights):
        accumulated += float(weight) / total
        if accumulated >= threshold:
            return position + 1
    return len(weights)


def adaptive_keep(inds, scores, threshold: float, min_keep: int = 1):
    """Adaptive top-k (``adaptive_topk.py:107-118``, ``:224-233``) on slots in
    descending order: per token keep = max(min(min_keep, k), keep_for_mass);
    slots past it name the token's first expert with score 0.  Returns the
    new ids, the masked scores and the keep counts.  Threshold 1.0 or more
    keeps every slot."""
    inds = np.array(inds)
    scores = f32(scores).copy()
    T, k = inds.shape
    keeps = np.full(T, k, dtype=np.int64)
    if threshold < 1.0:
        lo = max(1, min(k, int(min_keep)))
        for t in range(T):
            keep = max(lo, keep_for_mass(scores[t], threshold))
            keeps[t] = keep
            inds[t, keep:] = inds[t, 0]
            scores[t, keep:] = 0.0
    return inds, scores, keeps


def router(x, wg, k: int, logits=None, bias=None, threshold: float = 1.0, min_keep: int = 1) -> RouterOut:
    """Router chain of ``adaptive_topk.py:59-65`` plus renorm ``:257-262``.

    ``logits`` may be supplied (e.g. the device's own logits) to check the
    softmax/top-k stage on identical inputs.  ``bias`` ([E], bf16 values) is
    added to the bf16 logits before softmax/top-k and the sum rounded to bf16
    (the skewed-load benchmark's +2.0 on hot experts); supplied logits are
    taken as already biased.  ``threshold`` < 1.0 runs adaptive top-k
    (``adaptive_keep``): the top-k mass stays the sum over every slot, the
    renorm divides by the kept mass (blend 1.0).  The slots are in descending
    logit order (ties by expert id), a descending order of the bf16
    probabilities; the reference sorts its scores with argsort, whose order
    among equal bf16 probabilities is its own.
    """
    if logits is None:
        logits = router_logits(x, wg)
        if bias is not None:
            logits = bf16_round(f32(bf16_round(logits)) + f32(bias)[None, :])
    logits = bf16_round(logits)
    probs = softmax_bf16(logits)
    inds = topk_order(logits, k)
    scores = np.take_along_axis(probs, inds, axis=-1)
    mass = bf16_round(scores.sum(axis=-1, keepdims=True, dtype=np.float32))
    inds, kept, _ = adaptive_keep(inds, scores, threshold, min_keep)
    weights = renorm(kept, mass, 1.0)
    return RouterOut(logits, probs, inds, kept, mass, weights)


# --------------------------------------------------------------------------
# Permutation (mlx-vlm _gather_sort / _scatter_unsort)
# --------------------------------------------------------------------------


def gather_sort(inds, num_experts: int | None = None):
    """Stable sort of the flat (token, slot) list by expert id.

    Returns ``order`` (flat pair index at each sorted position), ``inverse``
    (sorted position of each flat pair), ``sorted_experts`` and
    ``offsets`` [E+1] (start of each expert's run).
    """
    flat = np.asarray(inds).reshape(-1).astype(np.int64)
    order = np.argsort(flat, kind="stable").astype(np.int32)
    inverse = np.empty_like(order)
    inverse[order] = np.arange(order.size, dtype=np.int32)
    E = int(num_experts if num_experts is not None else (flat.max() + 1 if flat.size else 0))
    counts = np.bincount(flat, minlength=E)[:E] if flat.size else np.zeros(E, np.int64)
    offsets = np.zeros(E + 1, dtype=np.int32)
    offsets[1:] = np.cumsum(counts)
    return order, inverse, flat[order].astype(np.int32), offsets


# --------------------------------------------------------------------------
# Whole block
# --------------------------------------------------------------------------


@dataclass
class Q4Bank:
    """Packed projection weights ``w`` [E, out, in/8] with bf16 scales/biases
    [E, out, in/group] (float32 arrays holding bf16 values)."""

    w: np.ndarray
    scales: np.ndarray
    biases: np.ndarray

    def expert(self, e: int) -> "Q4Bank":
        return Q4Bank(self.w[e], self.scales[e], self.biases[e])


@dataclass
class MoEParams:
    gate: Q4Bank            # [E, I, d/8]
    up: Q4Bank              # [E, I, d/8]
    down: Q4Bank            # [E, d, I/8]
    router_w: np.ndarray    # bf16 [E, d]
    shared_gate: Q4Bank     # [1, Is, d/8]
    shared_up: Q4Bank
    shared_down: Q4Bank     # [1, d, Is/8]
    shared_expert_gate: Q4Bank  # [1, 1, d/8]
    top_k: int = 10
    group_size: int = GROUP_SIZE

    @property
    def num_experts(self) -> int:
        return self.gate.w.shape[0]

    @property
    def hidden(self) -> int:
        return self.down.w.shape[1]


def _proj_bf16(x, bank: Q4Bank, group_size):
    return bf16_round(qmv(x, bank.w, bank.scales, bank.biases, group_size).astype(np.float32))


def expert_mlp_bf16(x, gate: Q4Bank, up: Q4Bank, down: Q4Bank, group_size=GROUP_SIZE):
    """One expert's bf16 path: gate/up projections (bf16 out), bf16 SwiGLU,
    down projection (bf16 out).  Returns (g, u, h, y)."""
    g = _proj_bf16(x, gate, group_size)
    u = _proj_bf16(x, up, group_size)
    h = silu_mul_bf16(g, u)
    y = _proj_bf16(h, down, group_size)
    return g, u, h, y


def dequantize_bf16(bank: Q4Bank, group_size=GROUP_SIZE) -> np.ndarray:
    """Weights as MLX's quantized-matmul kernels stage them for large batches:
    ``bf16(scale*q + bias)``, one rounding of the exact value (the float32
    product ``scale*q`` is exact; the sum with the bias then rounds once)."""
    return bf16_round(dequantize(bank.w, bank.scales, bank.biases, group_size))


def qmm_bf16(x, bank: Q4Bank, group_size=GROUP_SIZE) -> np.ndarray:
    """The prefill-path projection (MLX ``gather_qmm`` on sorted, batched
    rows, expert_cache.py:2017-2037): bf16 dequantised tile, products summed
    in high precision, bf16 out.  The float64 sum stands in for the kernel's
    float32 tensor-core accumulation, whose order is the hardware's."""
    w = dequantize_bf16(bank, group_size).astype(np.float64)
    return bf16_round((f32(x).astype(np.float64) @ w.T).astype(np.float32))


def expert_mlp_qmm(x, gate: Q4Bank, up: Q4Bank, down: Q4Bank, group_size=GROUP_SIZE):
    """One expert on the prefill path: bf16-dequantised gate/up and down
    tiles, bf16 SwiGLU between.  Returns (g, u, h, y)."""
    g = qmm_bf16(x, gate, group_size)
    u = qmm_bf16(x, up, group_size)
    h = silu_mul_bf16(g, u)
    y = qmm_bf16(h, down, group_size)
    return g, u, h, y


def shared_parts(x, p: MoEParams, path: str = "decode"):
    """``shared = shared_expert(x)``, ``sg = sigmoid(shared_expert_gate(x))``
    in bf16 (``adaptive_topk.py:264-265``).  ``path="prefill"`` computes the
    shared expert as the batched quantized matmul does (:func:`expert_mlp_qmm`);
    the gate row is a single-row product either way."""
    mlp = expert_mlp_qmm if path == "prefill" else expert_mlp_bf16
    _, _, _, shared = mlp(
        x, p.shared_gate.expert(0), p.shared_up.expert(0), p.shared_down.expert(0),
        p.group_size)
    z = _proj_bf16(x, p.shared_expert_gate.expert(0), p.group_size)   # [T, 1]
    sg = sigmoid_bf16(z)
    return shared, sg


def routed_outputs(x, inds, p: MoEParams, path: str = "decode"):
    """Per-(token, slot) bf16 down outputs [T, k, d], computing each distinct
    expert once for all of its tokens (the sorted gather_qmm pass).
    ``path="prefill"`` uses the batched quantized matmul's arithmetic
    (:func:`expert_mlp_qmm`), the decode default MLX's qmv formula."""
    mlp = expert_mlp_qmm if path == "prefill" else expert_mlp_bf16
    x = f32(x)
    T, k = inds.shape
    out = np.zeros((T, k, p.hidden), dtype=np.float32)
    hs = np.zeros((T, k, p.up.w.shape[1]), dtype=np.float32)
    flat = inds.reshape(-1)
    for e in np.unique(flat):
        pairs = np.nonzero(flat == e)[0]
        toks = pairs // k
        _, _, h, y = mlp(x[toks], p.gate.expert(e), p.up.expert(e), p.down.expert(e),
                         p.group_size)
        out.reshape(T * k, -1)[pairs] = y
        hs.reshape(T * k, -1)[pairs] = h
    return out, hs


def fused_combine(yd, weights, shared_y) -> np.ndarray:
    """``metal_runtime.py:315-334``: float32 accumulation of
    ``float(bf16(y_s)) * score_s`` in slot order with no fused multiply-add,
    then ``bf16(float(bf16(acc)) + float(shared_y))``."""
    yd = f32(yd)
    w = f32(weights)
    T, k, d = yd.shape
    acc = np.zeros((T, d), dtype=np.float32)
    for s in range(k):
        prod = (yd[:, s, :] * w[:, s:s + 1]).astype(np.float32)
        acc = (acc + prod).astype(np.float32)
    routed = bf16_round(acc)
    if shared_y is None:
        return routed
    return bf16_round(routed + f32(shared_y))


def generic_combine(yd, weights, shared, sg) -> np.ndarray:
    """``adaptive_topk.py:275-278`` in bf16: products rounded to bf16, summed
    in float32, rounded; plus ``bf16(sg*shared)``."""
    prods = bf16_round(f32(yd) * f32(weights)[..., None])
    y = bf16_round(prods.sum(axis=-2, dtype=np.float32))
    return bf16_round(y + bf16_round(f32(sg) * f32(shared)))


@dataclass
class BlockOut:
    y: np.ndarray
    router: RouterOut
    shared: np.ndarray
    sg: np.ndarray
    shared_y: np.ndarray
    yd: np.ndarray
    h: np.ndarray = field(repr=False, default=None)


def moe_block(x, p: MoEParams, semantics: str = "fused", logits=None,
              path: str = "decode", threshold: float = 1.0, min_keep: int = 1) -> BlockOut:
    """The routed sparse-MoE block ``_moe_call`` (``adaptive_topk.py:54-293``)
    at blend 1.0; ``threshold`` < 1.0 runs adaptive top-k (``router``).

    ``semantics="fused"`` is the custom-executor combine (float32); the
    ``"generic"`` form is the bf16 combine of the MLX path.  ``path`` picks the
    expert arithmetic: ``"decode"`` (MLX's qmv, the custom executor's few-row
    regime) or ``"prefill"`` (the sorted batched quantized matmul of
    ``expert_cache.py:2017-2037``, bf16-dequantised tiles).
    """
    x = bf16_round(x)
    r = router(x, p.router_w, p.top_k, logits=logits, threshold=threshold, min_keep=min_keep)
    shared, sg = shared_parts(x, p, path)
    shared_y = bf16_round(sg * shared)
    yd, h = routed_outputs(x, r.inds, p, path)
    if semantics == "fused":
        y = fused_combine(yd, r.weights, shared_y)
    elif semantics == "generic":
        y = generic_combine(yd, r.weights, shared, sg)
    else:
        raise ValueError(semantics)
    return BlockOut(y, r, shared, sg, shared_y, yd, h)


def keeps_of(inds) -> np.ndarray:
    """Keep counts of an adaptive routing (``adaptive_keep``): a token's top-k
    ids are distinct, so the first slot after slot 0 that repeats slot 0's
    expert is the first dropped one."""
    inds = np.asarray(inds)
    T, k = inds.shape
    keeps = np.full(T, k, dtype=np.int64)
    for t in range(T):
        rep = np.nonzero(inds[t, 1:] == inds[t, 0])[0]
        if rep.size:
            keeps[t] = int(rep[0]) + 1
    return keeps


def moe_block_reference_f64(x, p: MoEParams, inds, logits, keeps=None) -> np.ndarray:
    """Unrounded reference of the block for a fixed routing: every stage in
    float64 from the same bf16 inputs and bf16 router logits.  This is the
    "fp32 reference" that final outputs are compared with.  ``keeps``
    (adaptive top-k): slots past a token's count weigh nothing and the
    weights renormalise over the kept ones."""
    x = f32(x).astype(np.float64)
    l = f32(logits).astype(np.float64)
    e = np.exp(l - l.max(axis=-1, keepdims=True))
    probs = e / e.sum(axis=-1, keepdims=True)
    sc = np.take_along_axis(probs, inds, axis=-1)
    if keeps is not None:
        sc = sc * (np.arange(inds.shape[1])[None, :] < np.asarray(keeps)[:, None])
    w = sc / sc.sum(axis=-1, keepdims=True)

    def mlp(xx, gate, up, down):
        g = qmv(xx, gate.w, gate.scales, gate.biases, p.group_size)
        u = qmv(xx, up.w, up.scales, up.biases, p.group_size)
        h = g / (1.0 + np.exp(-g)) * u
        return qmv(h, down.w, down.scales, down.biases, p.group_size)

    T, k = inds.shape
    y = np.zeros((T, p.hidden))
    flat = inds.reshape(-1)
    for ex in np.unique(flat):
        pairs = np.nonzero(flat == ex)[0]
        toks = pairs // k
        yy = mlp(x[toks], p.gate.expert(ex), p.up.expert(ex), p.down.expert(ex))
        np.add.at(y, toks, yy * w.reshape(-1)[pairs][:, None])
    shared = mlp(x, p.shared_gate.expert(0), p.shared_up.expert(0), p.shared_down.expert(0))
    z = qmv(x, p.shared_expert_gate.w[0], p.shared_expert_gate.scales[0],
            p.shared_expert_gate.biases[0], p.group_size)
    sg = 1.0 / (1.0 + np.exp(-z))
    return y + sg * shared


def executor_reference_all(x, routes, gate: Q4Bank, up: Q4Bank, down: Q4Bank,
                           hidden_size: int, group_size: int = GROUP_SIZE):
    """The reference executor's NumPy path (``metal_runtime.py:976-983``):
    projections by :func:`numpy_projection` and a float32 SiLU written as
    ``up * (gate / (1 + exp(-gate)))``."""
    x = np.asarray(x)
    g = numpy_projection(x, routes, gate.w, gate.scales, gate.biases,
                         gate.w.shape[1], False, group_size)
    u = numpy_projection(x, routes, up.w, up.scales, up.biases,
                         up.w.shape[1], False, group_size)
    act = u * (g / (1.0 + np.exp(-g)))
    d = numpy_projection(act, routes, down.w, down.scales, down.biases,
                         hidden_size, True, group_size)
    return g, u, d


def rms_norm(x, gain, eps: float = 1e-6) -> np.ndarray:
    """``patch_rmsnorm.py:117-120``: float32 ``x*rsqrt(mean(x^2)+eps)*gain``,
    cast to bf16."""
    xf = f32(x)
    ms = np.mean(np.square(xf), axis=-1, keepdims=True, dtype=np.float32)
    r = (np.float32(1) / np.sqrt(ms + np.float32(eps))).astype(np.float32)
    return bf16_round(xf * r * f32(gain))


def weighted_combine(expert_outputs, routes, scores):
    """NumPy form of the reference's ``weighted_combine``
    (``metal_runtime.py:145-191``): select slots when the outputs hold every
    expert, then ``sum(selected * scores[..., None], axis=-2)``."""
    out = np.asarray(expert_outputs)
    routes = np.asarray(routes)
    scores = np.asarray(scores)
    if out.ndim < 2 or routes.ndim == 0:
        raise ValueError("expert_outputs and routes need at least one dimension")
    if scores.shape != routes.shape:
        raise ValueError("routes and scores must have identical shapes")
    if out.shape[:-1] == routes.shape:
        sel = out
    elif out.ndim == routes.ndim + 1 and out.shape[-2] >= routes.shape[-1]:
        if routes.size and (routes.min() < 0 or routes.max() >= out.shape[-2]):
            raise ValueError("routes contain an expert outside expert_outputs")
        sel = np.take_along_axis(out, routes[..., None], axis=-2)
    else:
        raise ValueError(
            f"expert_outputs shape {out.shape} does not match routes {routes.shape}")
    return (sel * scores[..., None]).sum(axis=-2)


# --------------------------------------------------------------------------
# Tiled expert pool (this build's resident record layout)
# --------------------------------------------------------------------------
#
# The reference keeps each expert as one fixed-stride record holding the MLX
# arrays (slab_pack.py:1-25).  The B200 pool re-tiles the same bytes so one
# bulk copy brings a warp everything it needs for 128 inputs of a row tile.
# These two functions restate that layout on the CPU so the packing kernel is
# checked byte for byte and the round trip back to the MLX arrays is exact.


def tile_records(a: Q4Bank, b: Q4Bank | None = None, tile_rows: int = 16,
                 group_size: int = GROUP_SIZE) -> np.ndarray:
    """Records of bank `a` (and `b`, the up half of a gate/up pair) as uint8:
    per (expert, row tile, 128-input chunk) the packed words [p][m][h][g][c]
    (4 words each; row 16m+g+8h, words 4c..4c+3 of the chunk), then the
    scales/biases.  Groups of 32: [p][m][g][c&1][h]{s_a, s_b, b_a, b_b} of
    groups 4ch+2(c&1) and +1.  Groups of 64 (kept as stored):
    [p][m][g][cb][h]{s, b} of group 2ch+cb.  Out-of-range rows and groups are
    zero."""
    if group_size not in (32, 64):
        raise ValueError("tiled records hold groups of 32 or 64")
    banks = [a] if b is None else [a, b]
    E, out, W = a.w.shape
    K = W * 8
    G = K // group_size
    MT = tile_rows // 16
    RB = -(-out // tile_rows)
    nch = -(-K // 128)
    gpc = 128 // group_size          # groups per 128-input chunk
    wparts, sparts = [], []
    for bk in banks:
        w = np.zeros((E, RB * tile_rows, nch * 16), np.uint32)
        w[:, :out, :W] = bk.w
        # [E, RB, MT, h, g, nch, c, j] -> [E, RB, nch, MT, h, g, c, j]
        w = w.reshape(E, RB, MT, 2, 8, nch, 4, 4).transpose(0, 1, 5, 2, 3, 4, 6, 7)
        wparts.append(w.reshape(E, RB, nch, MT, 1024 // 4))
        sb = np.zeros((2, E, RB * tile_rows, nch * gpc), np.uint16)
        sb[0, :, :out, :G] = bf16_bits(bk.scales)
        sb[1, :, :out, :G] = bf16_bits(bk.biases)
        if group_size == 32:
            # [kind, E, RB, MT, h, g, nch, cb, ab] -> [E, RB, nch, MT, g, cb, h, kind, ab]
            sb = sb.reshape(2, E, RB, MT, 2, 8, nch, 2, 2).transpose(1, 2, 6, 3, 5, 7, 4, 0, 8)
        else:
            # [kind, E, RB, MT, h, g, nch, cb] -> [E, RB, nch, MT, g, cb, h, kind]
            sb = sb.reshape(2, E, RB, MT, 2, 8, nch, 2).transpose(1, 2, 6, 3, 5, 7, 4, 0)
        sparts.append(sb.reshape(E, RB, nch, MT, -1))
    wcat = np.concatenate(wparts, axis=3).view(np.uint8).reshape(E, RB, nch, -1)
    scat = np.concatenate(sparts, axis=3).view(np.uint8).reshape(E, RB, nch, -1)
    return np.ascontiguousarray(np.concatenate([wcat, scat], axis=3)).reshape(-1)


def untile_records(rec: np.ndarray, experts: int, out: int, inn: int, nproj: int,
                   tile_rows: int, group_size: int = GROUP_SIZE
                   ) -> list[tuple[np.ndarray, np.ndarray, np.ndarray]]:
    """Inverse of tile_records: per projection (w uint32 [E, out, in/8], scale
    bits, bias bits uint16 [E, out, in/group_size])."""
    MT = tile_rows // 16
    RB = -(-out // tile_rows)
    nch = -(-inn // 128)
    sbytes = 256 if group_size == 32 else 128
    per = nproj * MT * (1024 + sbytes)
    r = np.asarray(rec, np.uint8).reshape(experts, RB, nch, per)
    wb = np.ascontiguousarray(r[..., :nproj * MT * 1024]).view(np.uint32)
    sbb = np.ascontiguousarray(r[..., nproj * MT * 1024:]).view(np.uint16)
    wb = wb.reshape(experts, RB, nch, nproj, MT, 2, 8, 4, 4)
    res = []
    for p in range(nproj):
        w = wb[:, :, :, p].transpose(0, 1, 3, 4, 5, 2, 6, 7).reshape(experts, RB * tile_rows, nch * 16)
        if group_size == 32:
            sp = sbb.reshape(experts, RB, nch, nproj, MT, 8, 2, 2, 2, 2)[:, :, :, p]
            # [E, RB, nch, MT, g, cb, h, kind, ab] -> [kind, E, RB, MT, h, g, nch, cb, ab]
            s = sp.transpose(7, 0, 1, 3, 6, 4, 2, 5, 8).reshape(2, experts, RB * tile_rows, nch * 4)
        else:
            sp = sbb.reshape(experts, RB, nch, nproj, MT, 8, 2, 2, 2)[:, :, :, p]
            # [E, RB, nch, MT, g, cb, h, kind] -> [kind, E, RB, MT, h, g, nch, cb]
            s = sp.transpose(7, 0, 1, 3, 6, 4, 2, 5).reshape(2, experts, RB * tile_rows, nch * 2)
        G = inn // group_size
        res.append((w[:, :out, :inn // 8], s[0, :, :out, :G], s[1, :, :out, :G]))
    return res


# --------------------------------------------------------------------------
# Synthetic inputs (seeded; the distributions of the benchmark configs)
# --------------------------------------------------------------------------


def make_q4_bank(rng, experts, out_w, in_w, group_size=GROUP_SIZE) -> Q4Bank:
    """Codes uniform in 0..15 (uniform uint32 words), scale =
    bf16(|N(0,0.02)|/8), bias = -8*scale (exact in bf16)."""
    w = rng.integers(0, 2**32, size=(experts, out_w, in_w // 8), dtype=np.uint32)
    s = bf16_round(np.abs(rng.normal(0.0, 0.02, size=(experts, out_w, in_w // group_size))) / 8)
    b = (np.float32(-8) * s).astype(np.float32)
    return Q4Bank(w, s, b)


def make_params(seed=0, experts=512, hidden=2048, inter=512, shared_inter=512,
                top_k=10, group_size=GROUP_SIZE) -> MoEParams:
    rng = np.random.default_rng(seed)
    gate = make_q4_bank(rng, experts, inter, hidden, group_size)
    up = make_q4_bank(rng, experts, inter, hidden, group_size)
    down = make_q4_bank(rng, experts, hidden, inter, group_size)
    router_w = bf16_round(rng.normal(0.0, 0.02, size=(experts, hidden)))
    sh_gate = make_q4_bank(rng, 1, shared_inter, hidden, group_size)
    sh_up = make_q4_bank(rng, 1, shared_inter, hidden, group_size)
    sh_down = make_q4_bank(rng, 1, hidden, shared_inter, group_size)
    seg = make_q4_bank(rng, 1, 1, hidden, group_size)
    return MoEParams(gate, up, down, router_w, sh_gate, sh_up, sh_down, seg, top_k, group_size)


def make_x(seed, tokens, hidden) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return bf16_round(rng.normal(0.0, 1.0, size=(tokens, hidden)))


# --------------------------------------------------------------------------
# Comparison helpers used by the tests
# --------------------------------------------------------------------------


def max_rel_error(actual, ref, floor_frac: float = 0.05) -> float:
    """max |a-r| / max(|r|, floor) with floor = floor_frac * rms(r)."""
    a = np.asarray(actual, dtype=np.float64)
    r = np.asarray(ref, dtype=np.float64)
    if a.shape != r.shape:
        raise ValueError(f"shape mismatch {a.shape} vs {r.shape}")
    if r.size == 0:
        return 0.0
    floor = floor_frac * float(np.sqrt(np.mean(r * r))) + 1e-30
    return float(np.max(np.abs(a - r) / np.maximum(np.abs(r), floor)))


def summand_scale(yd, weights, shared_y=None) -> np.ndarray:
    """Per-output magnitude of the terms a block output sums:
    ``sum_s |w_s * y_s| + |shared_y|`` [T, d].  The rounding error of a sum
    is bounded relative to this (not to the sum itself, which may cancel),
    so it is the natural denominator floor of a max-relative-error check."""
    s = np.abs(f32(yd).astype(np.float64) * f32(weights).astype(np.float64)[..., None]).sum(axis=-2)
    if shared_y is not None:
        s = s + np.abs(f32(shared_y).astype(np.float64))
    return s


def max_rel_error_floored(actual, ref, floor) -> float:
    """max |a-r| / max(|r|, floor) with a per-element floor array."""
    a = np.asarray(actual, dtype=np.float64)
    r = np.asarray(ref, dtype=np.float64)
    if r.size == 0:
        return 0.0
    den = np.maximum(np.abs(r), np.asarray(floor, dtype=np.float64)) + 1e-30
    return float(np.max(np.abs(a - r) / den))


def normwise_error(actual, ref) -> float:
    a = np.asarray(actual, dtype=np.float64)
    r = np.asarray(ref, dtype=np.float64)
    den = float(np.max(np.abs(r))) if r.size else 0.0
    return float(np.max(np.abs(a - r)) / den) if den else float(np.max(np.abs(a - r), initial=0.0))


__all__ = [name for name in dir() if not name.startswith("_")]
