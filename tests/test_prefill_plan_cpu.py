"""Chunk plan and layer-major windows (vxmoe.prefill), the rules of
models/flashnext/prefill.py:109-207 and layer_major.py:155-186."""
from __future__ import annotations

import pytest

from vxmoe import prefill as P


def test_grid_edges_and_short_tail_merge():
    assert P.plan_chunks(5000, 2048) == [(0, 2048), (2048, 4096), (4096, 5000)]
    # a 34-token tail would run decode-shaped kernels: merged into the chunk before
    assert P.plan_chunks(4130, 2048) == [(0, 2048), (2048, 4130)]
    # ... unless its edge is a requested boundary
    assert P.plan_chunks(4130, 2048, boundaries=[4100]) == [(0, 2048), (2048, 4096), (4096, 4100),
                                                            (4100, 4130)]
    assert P.plan_chunks(0, 2048) == []
    assert P.plan_chunks(100, 0) == [(0, 100)]


@pytest.mark.parametrize("policy", ["grid", "balanced"])
def test_resumed_run_continues_the_cold_plan(policy):
    """A run restored at an edge of the cold plan (offset tokens already
    cached) takes exactly the cold run's remaining spans."""
    total, chunk, anchors = 9000, 2048, [700, 5100]
    cold = P.plan_chunks(total, chunk, boundaries=anchors, policy=policy)
    for a, _ in cold[1:]:
        tail = P.plan_chunks(total - a, chunk, boundaries=anchors, offset=a, policy=policy)
        assert [(s + a, e + a) for s, e in tail] == [sp for sp in cold if sp[0] >= a]


def test_balanced_pieces():
    assert P.plan_chunks(5000, 2048, policy="balanced") == [(0, 1667), (1667, 3334), (3334, 5000)]
    assert P.plan_chunks(5000, 2048, boundaries=[1000], policy="balanced") == [(0, 1000), (1000, 3000),
                                                                                (3000, 5000)]
    spans = P.plan_chunks(10_001, 2048, policy="balanced")
    sizes = [e - s for s, e in spans]
    assert max(sizes) <= 2048 and max(sizes) - min(sizes) <= 1 and sum(sizes) == 10_001


def test_windows():
    spans = [(0, 2048), (2048, 4096), (4096, 6144), (6144, 8192), (8192, 9000)]
    assert P.plan_windows(spans, 0, 4096) == [spans[0:2], spans[2:4], spans[4:5]]
    # a required position ends the window where it falls
    assert P.plan_windows(spans, 0, 8192, required=[4096]) == [spans[0:2], spans[2:5]]
    # an anchor past the window's middle is preferred to the last edge that fits
    assert P.plan_windows(spans, 0, 8192, anchors=[6144]) == [spans[0:3], spans[3:5]]
    # a chunk larger than the window forms its own window
    assert P.plan_windows([(0, 5000), (5000, 6000)], 0, 4096) == [[(0, 5000)], [(5000, 6000)]]


def test_bad_policy_and_sizes():
    with pytest.raises(ValueError):
        P.plan_chunks(100, 64, policy="budgeted")
    with pytest.raises(ValueError):
        P.plan_chunks(-1, 64)


# Budgeted policy (prefill.py:109-140): a model whose attention term grows with
# the position, so the chunks shrink along the prompt.
_MODEL = P.ChunkMemoryModel(per_token=100_000, pair_bytes=48, query_cap=2048)


def test_budgeted_chunks_shrink_with_position():
    # 2048 fits while 2048*1e5 + 2048*(p+2048)*48 <= 1e9, i.e. p <= 6041;
    # 1024 while p <= 17237; then 512.
    spans = P.plan_chunks(20_000, 0, policy="budgeted", budget=10**9, model=_MODEL)
    sizes = [e - s for s, e in spans]
    assert sizes == [2048] * 3 + [1024] * 11 + [512] * 4 + [544]   # 32-token tail merged
    for s, e in spans[:-1]:
        assert _MODEL.increment(e - s, s) <= 10**9
    # a cap below the largest candidate
    assert {e - s for s, e in P.plan_chunks(3000, 1024, policy="budgeted", budget=10**9,
                                              model=_MODEL)[:-1]} == {1024}


def test_budgeted_anchors_tiny_budget_and_resume():
    anchors = [700, 5100]
    cold = P.plan_chunks(9000, 0, boundaries=anchors, policy="budgeted", budget=10**9, model=_MODEL)
    assert (0, 700) in cold and any(e == 5100 for _, e in cold)
    for a, _ in cold[1:]:
        tail = P.plan_chunks(9000 - a, 0, boundaries=anchors, offset=a, policy="budgeted",
                             budget=10**9, model=_MODEL)
        assert [(s + a, e + a) for s, e in tail] == [sp for sp in cold if sp[0] >= a]
    # nothing fits: the smallest candidate everywhere
    huge = P.ChunkMemoryModel(per_token=10**7)
    spans = P.plan_chunks(1000, 0, policy="budgeted", budget=10**8, model=huge)
    assert [e - s for s, e in spans] == [256, 256, 256, 232]
    with pytest.raises(ValueError):
        P.plan_chunks(1000, 0, policy="budgeted", budget=10**6, model=huge)



def test_plans_match_the_reference_planner():
    """Golden plans written by the reference's own planner (make_prefill_golden.py):
    grid, balanced and budgeted, cold and resumed; the budgeted ones with the
    reference's estimate expressed as a ChunkMemoryModel."""
    import json
    import os
    d = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "prefill_plans.json")))
    assert tuple(d["candidates"]) == P.CANDIDATE_CHUNKS
    est = d["estimate"]
    model = P.ChunkMemoryModel(per_token=est["per_token"], pair_bytes=est["pair_bytes"],
                               query_cap=est["query_cap"], kv_per_token=est["kv_per_token"])
    for c in d["cases"]:
        kw = dict(boundaries=c["boundaries"], offset=c["offset"], policy=c["policy"], anchors=c["anchors"])
        if c["policy"] == "budgeted":
            kw.update(budget=c["budget"], model=model)
        got = P.plan_chunks(c["total"], c["chunk"], **kw)
        assert [list(s) for s in got] == c["spans"], c


def test_windows_match_the_reference_planner():
    """Golden layer-major windows from the reference's plan_windows
    (layer_major.py:155-186), required positions and anchors included."""
    import json
    import os
    d = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "prefill_plans.json")))
    assert d["windows"]
    for w in d["windows"]:
        spans = [tuple(s) for s in w["spans"]]
        got = P.plan_windows(spans, w["offset"], w["window"], w["required"], w["anchors"])
        assert [[list(s) for s in g] for g in got] == w["groups"], w
