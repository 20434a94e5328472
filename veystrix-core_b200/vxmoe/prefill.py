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

import bisect
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
    """The chunk the budgeted policy takes at `position`: the largest
    candidate size not above `cap` whose memory increment there fits the
    budget, else the smallest size allowed (prefill.py:109-117)."""
    sizes = sorted((c for c in CANDIDATE_CHUNKS if c <= cap), reverse=True)
    if not sizes:
        sizes = [min(CANDIDATE_CHUNKS)]
    fitting = (c for c in sizes if model.increment(c, position) <= budget)
    return next(fitting, sizes[-1])


# -- one walk for every policy ------------------------------------------------
#
# A plan is the list of cut positions a walk from position 0 to the prompt's
# end makes.  Each policy is a step function: the policy's next cut after a
# position (the walk never steps past an anchor, so a step only needs the
# anchor-bounded segment it starts in).  Anchors are cuts of every policy.
# Because each cut depends only on the position it is taken from, the cuts
# after any cut of the cold plan are the same whether the walk starts at 0
# or there: a run resumed at a cut takes the cold run's remaining spans.

Step = Callable[[int, int], int]   # (position, segment end) -> next cut (may pass the segment end)


def _walk(end: int, step: Step, anchors: Sequence[int], merge_short_tail: bool) -> List[int]:
    """Cuts in (0, end) of the walk: at each position the nearer of the
    policy's next cut and the next anchor.  With `merge_short_tail` a last
    piece shorter than MIN_CHUNK_TOKENS joins the one before it, unless the
    cut before it is an anchor."""
    stops = sorted({int(a) for a in anchors if 0 < int(a) < end})
    cuts: List[int] = []
    pos, k = 0, 0
    while pos < end:
        while k < len(stops) and stops[k] <= pos:
            k += 1
        seg_end = stops[k] if k < len(stops) else end
        nxt = min(step(pos, seg_end), seg_end)
        if nxt <= pos:
            raise RuntimeError("chunk plan made no progress")
        if nxt < end:
            cuts.append(nxt)
        pos = nxt
    if merge_short_tail and cuts and end - cuts[-1] < MIN_CHUNK_TOKENS and cuts[-1] not in stops:
        cuts.pop()
    return cuts


def _grid_step(chunk: int) -> Step:
    # the next multiple of the chunk size (absolute positions)
    return lambda pos, seg_end: (pos // chunk + 1) * chunk if chunk else seg_end


def _balanced_step(chunk: int, segment_start: Callable[[int], int]) -> Step:
    # a segment of n tokens in ceil(n / chunk) pieces as equal as integers
    # allow, the longer pieces first: the cut after `pos` is the first piece
    # boundary past it
    def step(pos: int, seg_end: int) -> int:
        lo = segment_start(pos)
        n = seg_end - lo
        pieces = -(-n // chunk) if chunk else 1
        size, longer = divmod(n, pieces)
        r = pos - lo
        if r < longer * (size + 1):                 # inside the longer pieces
            return lo + (r // (size + 1) + 1) * (size + 1)
        return lo + longer * (size + 1) + ((r - longer * (size + 1)) // size + 1) * size
    return step


def _budgeted_step(cap: int, budget: int, model: ChunkMemoryModel) -> Step:
    return lambda pos, seg_end: pos + budgeted_chunk(pos, cap, budget, model)


def budgeted_edges(end: int, cap: int, budget: int, model: ChunkMemoryModel,
                   anchors: Sequence[int] = ()) -> List[int]:
    """Cuts of the budgeted plan of a prompt ending at `end` (prefill.py:120-140)."""
    return _walk(end, _budgeted_step(cap, budget, model), anchors, True)


def balanced_edges(end: int, chunk: int, anchors: Sequence[int] = ()) -> List[int]:
    """Cuts of the balanced plan of a prompt ending at `end`."""
    marks = sorted({int(a) for a in anchors if 0 < int(a) < end})

    def segment_start(pos: int) -> int:
        return max([0] + [a for a in marks if a <= pos])

    return _walk(end, _balanced_step(chunk, segment_start), marks, False)


def plan_chunks(total: int, chunk: int, boundaries: Sequence[int] = (), offset: int = 0,
                policy: str = "grid", anchors: Optional[Sequence[int]] = None,
                budget: Optional[int] = None, model: Optional[ChunkMemoryModel] = None) -> List[Span]:
    """Spans [(start, end), ...] covering range(total) of a prompt whose first
    token sits at absolute position `offset` (tokens already in the cache).
    The grid policy cuts at `boundaries`; the other two at `anchors` (the
    boundaries when none are given).  The budgeted policy takes `budget`
    (bytes, at least MIN_BUDGET_BYTES) and the memory `model`; its cap is
    `chunk`, or the largest candidate when 0."""
    total, chunk, offset = int(total), int(chunk), int(offset)
    if total < 0 or chunk < 0 or offset < 0:
        raise ValueError("negative prompt length, chunk size or offset")
    end = offset + total
    marks = boundaries if anchors is None else anchors
    if policy == "grid":
        cuts = _walk(end, _grid_step(chunk), boundaries, True)
    elif policy == "balanced":
        cuts = balanced_edges(end, chunk, marks)
    elif policy == "budgeted":
        if budget is None or model is None:
            raise ValueError("the budgeted policy needs a budget and a memory model")
        if budget < MIN_BUDGET_BYTES:
            raise ValueError(f"chunk budget must be at least {MIN_BUDGET_BYTES} bytes")
        cuts = budgeted_edges(end, chunk or max(CANDIDATE_CHUNKS), int(budget), model, marks)
    else:
        raise ValueError(f"unknown chunk policy {policy!r} (grid, balanced or budgeted)")
    # the spans of this run: the cold plan's cuts after the cached prefix
    points = [offset] + [c for c in cuts if offset < c < end] + [end]
    return [(a - offset, b - offset) for a, b in zip(points, points[1:]) if b > a]


def plan_windows(spans: Sequence[Span], offset: int, window: int, required: Sequence[int] = (),
                 anchors: Sequence[int] = ()) -> List[List[Span]]:
    """Group consecutive chunk spans into layer-major windows of at most
    `window` tokens; a single larger chunk forms its own window.  A window
    ends at the first span end inside it that is a `required` position (a
    point the caller must observe between layers); otherwise, unless it
    already reaches the last span, at the last span end past its middle that
    is an `anchor`, else at the last span end that fits."""
    spans = [(int(a), int(b)) for a, b in spans]
    ends = [b for _, b in spans]
    must = [offset + b in set(int(p) for p in required) for b in ends]
    nice = [offset + b in set(int(p) for p in anchors) for b in ends]
    groups: List[List[Span]] = []
    first = 0
    while first < len(spans):
        start = spans[first][0]
        # the last span that still ends within the window (at least one span)
        last = max(first, bisect.bisect_right(ends, start + int(window), first) - 1)
        stop = next((m for m in range(first, last + 1) if must[m]), None)
        if stop is None:
            stop = last
            if last + 1 < len(spans):
                middle = start + int(window) // 2
                preferred = [m for m in range(first, last + 1) if nice[m] and ends[m] > middle]
                if preferred:
                    stop = preferred[-1]
        groups.append(spans[first:stop + 1])
        first = stop + 1
    return groups


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
