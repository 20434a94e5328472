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

Windows group whole chunks up to a token budget, ending at a required
position inside them, else at the last anchor past the window's middle, else
at the last chunk edge that fits.
"""
from __future__ import annotations

from typing import Callable, List, Optional, Sequence, Tuple

import torch

MIN_CHUNK_TOKENS = 64          # a shorter tail would run the decode-shaped kernels
Span = Tuple[int, int]


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
                policy: str = "grid", anchors: Optional[Sequence[int]] = None) -> List[Span]:
    """Spans [(start, end), ...] covering range(total) of a prompt whose first
    token sits at absolute position `offset` (tokens already in the cache)."""
    total, chunk, offset = int(total), int(chunk), int(offset)
    if total < 0 or chunk < 0 or offset < 0:
        raise ValueError("negative prompt length, chunk size or offset")
    end = offset + total
    if policy == "balanced":
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
        raise ValueError(f"unknown chunk policy {policy!r} (grid or balanced)")
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
