"""The reference benchmark's custom-executor slot driven through
``vxmoe.harness:build_executor`` the way models/flashnext/tests/bench/
bench_runtime_layer.py drives it: the target is called with only the context
names its signature takes (or all of them when it takes **kwargs,
``:110-140``), the runner's ``execute`` the same way (``:175-201``), with the
harness's context - x [1, 1, hidden], packs holding only the route's experts,
local indices [1, 1, width] and scores [1, 1, width] (``:383-410``) - and
the output compared with atol = rtol = 1e-2 (``:471-472``)."""
from __future__ import annotations

import inspect

import numpy as np
import pytest
import torch

import vxmoe_oracle as O

pytestmark = pytest.mark.gpu


def _call_by_signature(fn, values):
    """Call fn with the context entries its parameters name (everything when
    it takes **kwargs), as the reference harness's signature adapter does."""
    params = list(inspect.signature(fn).parameters.values())
    if any(p.kind == inspect.Parameter.VAR_KEYWORD for p in params):
        return fn(**values)
    kw = {p.name: values[p.name] for p in params
          if p.kind in (inspect.Parameter.POSITIONAL_OR_KEYWORD, inspect.Parameter.KEYWORD_ONLY)
          and p.name in values}
    return fn(**kw)


def _context(x, packs, width, scores, hidden):
    route = np.arange(width, dtype=np.int32)
    indices = route.reshape(1, 1, width)
    return {
        "x": x, "inputs": x, "hidden_states": x, "packs": packs, "weights": packs,
        "expert_weights": packs, "projections": packs, "gate": packs["gate_proj"],
        "up": packs["up_proj"], "down": packs["down_proj"], "gate_proj": packs["gate_proj"],
        "up_proj": packs["up_proj"], "down_proj": packs["down_proj"],
        "indices": indices, "rhs_indices": indices, "expert_indices": indices,
        "route": route, "expert_ids": route, "miss_fraction": 0.0, "miss": 0.0,
        "scores": scores, "gating_scores": scores,
        "routes": route.reshape(1, -1), "route_indices": route.reshape(1, -1),
        "expert_outputs": None, "expert_values": None,
        "group_size": 32, "bits": 4, "mode": "affine", "activation": None,
        "expert_count": width, "hidden_size": hidden, "top_k": width,
    }


@pytest.mark.parametrize("width,hidden,inter", [(8, 2048, 512), (10, 2560, 640)])
def test_harness_builds_and_runs_the_executor(width, hidden, inter):
    if not torch.cuda.is_available():
        pytest.fail("GPU tests need a CUDA device")
    from vxmoe import harness
    rng = np.random.default_rng(width)
    gate = O.make_q4_bank(rng, width, inter, hidden)
    up = O.make_q4_bank(rng, width, inter, hidden)
    down = O.make_q4_bank(rng, width, hidden, inter)
    packs = {n: (b.w, b.scales, b.biases) for n, b in
             (("gate_proj", gate), ("up_proj", up), ("down_proj", down))}
    x = O.make_x(width + 1, 1, hidden).reshape(1, 1, hidden)
    raw = rng.random(width).astype(np.float32)
    scores = O.bf16_round(raw / raw.sum()).reshape(1, 1, width)
    ctx = _context(x, packs, width, scores, hidden)
    runner = _call_by_signature(harness.build_executor, ctx)
    assert getattr(runner, "last_path", None) is None     # counted as the native path (:204-211)
    out = np.asarray(_call_by_signature(runner.execute, ctx))
    assert out.shape == (1, 1, hidden)
    # the harness's reference: each route's expert on x, weighted by its score
    routes = np.arange(width, dtype=np.int32).reshape(1, width)
    yd = np.zeros((1, width, hidden), np.float32)
    for s in range(width):
        _, _, _, yd[0, s] = O.expert_mlp_bf16(x.reshape(1, hidden), gate.expert(s), up.expert(s),
                                             down.expert(s))
    ref = O.fused_combine(yd, scores.reshape(1, width), None).reshape(1, 1, hidden)
    np.testing.assert_allclose(out, ref, atol=1e-2, rtol=1e-2)
    assert O.normwise_error(out, ref) < 1e-2
    # per-slot form: no scores in the context
    ctx_ns = dict(ctx, scores=None, gating_scores=None)
    slots = np.asarray(_call_by_signature(runner.execute, ctx_ns))
    assert slots.shape == (1, 1, width, hidden)
    np.testing.assert_allclose(slots.reshape(1, width, hidden), yd, atol=1e-2, rtol=1e-2)
    del routes
