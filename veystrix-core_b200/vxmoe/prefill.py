"""Prefill caller: the chunk plan and the layer-major window.

The reference cuts a prompt into chunks (models/flashnext/prefill.py:109-207)
and can run a window of several chunks layer-major - every layer over all of
the window's chunks before the next layer - so each layer's experts are read
once per window instead of once per chunk (layer_major.py:1-30, :155-186).
On B200 every expert is resident in HBM; the window is simply a larger batch
per layer for the tcgen05 grouped GEMM, which handles a token's product with
an expert independently of the other tokens in the batch, so the layer-major
result equals the chunk-major one bit for bit.

Plan rules (positions absolute, so a run resumed at an edge of the cold plan
continues with exactly the cold run's remaining spans):

* ``grid``: edges at every multiple of the chunk size and at each requested
  boundary; a last piece shorter than MIN_CHUNK_TOKENS is merged into the
  one before it unless that edge is a requested boundary.
* ``balanced``: between consecutive anchors, the fewest equal pieces of at
  most the chunk size, the first ``length % pieces`` pieces one token longer.
* ``budgeted``: greedy from position 0, each chunk the largest of
  CANDIDATE_CHUNKS (up to the cap) whose estimated device-memory increment at
  its start position fits the budget (the smallest when none fits), cut at
  anchors, with the grid rule's short-tail merge.  Each chunk depends only on
  its start position, so the plan is prefix-stable like the other two.

Windows group whole chunks up to a token budget, ending at a required
position inside them, else at the last anchor past the window's middle, else
at the last chunk edge that fits.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, List, Optional, Sequence, Tuple

import torch

MIN_CHUNK_TOKENS = 64          # a shorter tail would run the decode-shaped kernels
CANDIDATE_CHUNKS = (2048, 1024, 512, 256)   # largest first (prefill.py:45)
MIN_BUDGET_BYTES = 100_000_000               # prefill.py:104-105
Span = Tuple[int, int]


@dataclass(frozen=True)
class ChunkMemoryModel:
    """Device bytes a chunk of `chunk` tokens adds while it runs with
    `position` tokens already cached - the terms of the reference's estimate
    (prefill_budget.py:115-135): a transient per live token, attention scores
    for min(chunk, query_cap) queries against every key up to the chunk's end
    at `pair_bytes` per (query, key) pair, and the cache the chunk appends.
    `layer_bytes(chunk)` adds what one MoE-block call over the chunk takes
    (`block_memory_model`); the attention and cache terms belong to the model
    around the block and are the caller's to supply."""
    per_token: float = 0.0
    pair_bytes: float = 0.0
    query_cap: int = 2048
    kv_per_token: float = 0.0
    layer_bytes: Optional[Callable[[int], int]] = None

    def increment(self, chunk: int, position: int) -> int:
        chunk, position = int(chunk), int(position)
        scores = min(chunk, self.query_cap) * (position + chunk) * self.pair_bytes
        extra = self.layer_bytes(chunk) if self.layer_bytes is not None else 0
        return int(chunk * (self.per_token + self.kv_per_token) + scores + extra)


def block_memory_model(weights, **model) -> ChunkMemoryModel:
    """A ChunkMemoryModel whose layer term is this block's own device memory
    for a chunk: the library's scratch for one call (vx_moe_block_workspace)
    plus the output rows and the routes (ids int32, weights bf16)."""
    import ctypes

    from ._lib import load
    lib = load()
    st = weights.vx()
    row = weights.hidden * 2 + weights.top_k * (4 + 2)

    def layer_bytes(chunk: int) -> int:
        return int(lib.vx_moe_block_workspace(int(chunk), ctypes.byref(st))) + int(chunk) * row

    return ChunkMemoryModel(layer_bytes=layer_bytes, **model)


def budgeted_chunk(position: int, cap: int, budget: int, model: ChunkMemoryModel) -> int:
    """Largest candidate chunk <= cap whose increment at `position` fits the
    budget; the smallest candidate when none fits (prefill.py:109-117)."""
    cands = [c for c in CANDIDATE_CHUNKS if c <= cap] or [min(CANDIDATE_CHUNKS)]
    for c in cands:
        if model.increment(c, position) <= budget:
            return c
    return cands[-1]


def budgeted_edges(end: int, cap: int, budget: int, model: ChunkMemoryModel,
                   anchors: Sequence[int] = (), start: int = 0) -> List[int]:
    """Internal edges of the budgeted plan over [start, end] (prefill.py:120-140)."""
    wanted = sorted({int(a) for a in anchors if start < int(a) < end})
    edges: List[int] = []
    pos = int(start)
    while pos < end:
        stop = min(pos + budgeted_chunk(pos, cap, budget, model), end)
        cut = next((a for a in wanted if pos < a < stop), None)
        if cut is not None:
            stop = cut
        if stop < end:
            edges.append(stop)
        pos = stop
    if edges and end - edges[-1] < MIN_CHUNK_TOKENS and edges[-1] not in wanted:
        edges.pop()
    return edges


def balanced_edges(end: int, chunk: int, anchors: Sequence[int] = ()) -> List[int]:
    """Internal edges of the balanced cold plan over [0, end]."""
    points = [0] + sorted({int(a) for a in anchors if 0 < int(a) < end}) + [int(end)]
    edges: List[int] = []
    for lo, hi in zip(points, points[1:]):
        n = hi - lo
        pieces = -(-n // chunk) if chunk else 1
        size, extra = divmod(n, pieces)
        pos = lo
        for i in range(pieces):
            pos += size + (1 if i < extra else 0)
            edges.append(pos)
    return edges[:-1]


def plan_chunks(total: int, chunk: int, boundaries: Sequence[int] = (), offset: int = 0,
                policy: str = "grid", anchors: Optional[Sequence[int]] = None,
                budget: Optional[int] = None, model: Optional[ChunkMemoryModel] = None) -> List[Span]:
    """Spans [(start, end), ...] covering range(total) of a prompt whose first
    token sits at absolute position `offset` (tokens already in the cache).
    The budgeted policy takes `budget` (bytes, at least MIN_BUDGET_BYTES) and
    the memory `model`; its cap is `chunk`, or the largest candidate when 0."""
    total, chunk, offset = int(total), int(chunk), int(offset)
    if total < 0 or chunk < 0 or offset < 0:
        raise ValueError("negative prompt length, chunk size or offset")
    end = offset + total
    if policy == "budgeted":
        if budget is None or model is None:
            raise ValueError("the budgeted policy needs a budget and a memory model")
        if budget < MIN_BUDGET_BYTES:
            raise ValueError(f"chunk budget must be at least {MIN_BUDGET_BYTES} bytes")
        cold = budgeted_edges(end, chunk or max(CANDIDATE_CHUNKS), int(budget), model,
                              boundaries if anchors is None else anchors)
        points = [0] + [e - offset for e in cold if offset < e < end] + [total]
    elif policy == "balanced":
        cold = balanced_edges(end, chunk, boundaries if anchors is None else anchors)
        points = [0] + [e - offset for e in cold if offset < e < end] + [total]
    elif policy == "grid":
        edges = set(range((offset // chunk + 1) * chunk, end, chunk)) if chunk else set()
        wanted = {int(b) for b in boundaries if offset < int(b) < end}
        edges |= wanted
        ordered = sorted(edges)
        if ordered and end - ordered[-1] < MIN_CHUNK_TOKENS and ordered[-1] not in wanted:
            ordered.pop()
        points = [0] + [e - offset for e in ordered] + [total]
    else:
        raise ValueError(f"unknown chunk policy {policy!r} (grid, balanced or budgeted)")
    return [(a, b) for a, b in zip(points, points[1:]) if b > a]


def plan_windows(spans: Sequence[Span], offset: int, window: int, required: Sequence[int] = (),
                 anchors: Sequence[int] = ()) -> List[List[Span]]:
    """Group consecutive chunk spans into layer-major windows of at most
    `window` tokens (a single larger chunk forms its own window)."""
    spans = [(int(a), int(b)) for a, b in spans]
    req = {int(p) for p in required}
    anc = {int(p) for p in anchors}
    out: List[List[Span]] = []
    i = 0
    while i < len(spans):
        first = spans[i][0]
        limit = first + int(window)
        j = i
        while j + 1 < len(spans) and spans[j + 1][1] <= limit:
            j += 1
        forced = [m for m in range(i, j + 1) if offset + spans[m][1] in req]
        if forced:
            j = forced[0]
        elif j + 1 < len(spans):
            half = first + int(window) // 2
            nice = [m for m in range(i, j + 1) if offset + spans[m][1] in anc and spans[m][1] > half]
            if nice:
                j = nice[-1]
        out.append(spans[i:j + 1])
        i = j + 1
    return out


Layer = Callable[[torch.Tensor], torch.Tensor]


def run_chunk_major(layers: Sequence[Layer], x: torch.Tensor, spans: Sequence[Span]) -> torch.Tensor:
    """Every chunk through every layer, chunk by chunk."""
    out = torch.empty_like(x)
    for a, b in spans:
        h = x[a:b]
        for f in layers:
            h = f(h)
        out[a:b] = h
    return out


def run_layer_major(layers: Sequence[Layer], x: torch.Tensor, spans: Sequence[Span], window: int,
                    offset: int = 0, required: Sequence[int] = (), anchors: Sequence[int] = ()) -> torch.Tensor:
    """Each window of chunks through every layer as one batch per layer."""
    out = torch.empty_like(x)
    for group in plan_windows(spans, offset, window, required, anchors):
        a, b = group[0][0], group[-1][1]
        h = x[a:b]
        for f in layers:
            h = f(h)
        out[a:b] = h
    return out
