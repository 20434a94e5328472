"""Adapter for the reference's executor benchmark slot.

``tests/bench/bench_runtime_layer.py`` loads ``module:attribute`` with
``--custom-executor`` (``:85-100``), builds a runner by calling the target
with only the context names in its signature (``:112-172``) and then calls
``runner.execute`` the same way (``:175-201``).  Its context holds ``x``
[1, 1, hidden], ``packs`` {gate_proj, up_proj, down_proj: (weight, scales,
biases)}, ``indices`` [1, 1, width], ``scores`` [1, 1, width] and the
quantisation arguments (``:383-410``).  A runner without a ``last_path``
marker counts as a native run (``:204-211``), so this adapter has none.

    --custom-executor vxmoe.harness:build_executor
"""
from __future__ import annotations

import numpy as np
import torch

from . import ops


def _np(a):
    """Host copy of an MLX, NumPy or torch array (bf16 widened to float32)."""
    if isinstance(a, torch.Tensor):
        return a
    try:
        return np.asarray(a)
    except (TypeError, ValueError, RuntimeError):
        return np.asarray(a.astype(getattr(type(a), "float32", None) or _mx_float32()))


def _mx_float32():
    import mlx.core as mx  # only when the harness hands over MLX arrays
    return mx.float32


def _q4(triple, device):
    w, s, b = triple
    w = _np(w)
    if isinstance(w, np.ndarray):
        w = torch.from_numpy(np.ascontiguousarray(w.astype(np.uint32)))
    return ops.Q4Projection(w.to(device), ops._upload_bf16(_np(s), device),
                            ops._upload_bf16(_np(b), device))


class HarnessRunner:
    """Routed experts plus the score combine over the harness's packs."""

    def __init__(self, packs, top_k, device):
        self.device = device
        self.weights = ops.MoEWeights(_q4(packs["gate_proj"], device), _q4(packs["up_proj"], device),
                                      _q4(packs["down_proj"], device), top_k=top_k, device=device)

    def execute(self, x, indices, scores=None):
        shape = tuple(x.shape)
        xt = ops._upload_bf16(_np(x), self.device).reshape(-1, shape[-1])
        k = int(indices.shape[-1])
        r = ops._i32(_np(indices), self.device, "indices").reshape(-1, k)
        sc = None if scores is None else ops._upload_bf16(_np(scores), self.device).reshape(-1, k)
        out = ops.moe_experts(xt, r, self.weights, scores=sc)
        if sc is None:
            return out.reshape(*shape[:-1], k, shape[-1]).float().cpu().numpy()
        return out.reshape(shape).float().cpu().numpy()


def build_executor(packs, group_size=32, bits=4, mode="affine", top_k=None, **_ignored):
    if group_size != 32 or bits != 4 or mode != "affine":
        raise ValueError("vxmoe runs affine 4-bit group-32 weights")
    width = int(top_k) if top_k is not None else int(_np(packs["gate_proj"][0]).shape[0])
    return HarnessRunner(packs, width, torch.device("cuda"))
