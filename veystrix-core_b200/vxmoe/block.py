"""Block-level call surfaces of the reference's routed MoE layer.

``SwitchGLU`` mirrors ``StreamingSwitchGLU.__call__(x, indices, allow_sort,
scores, shared_y, shared, shared_gate)`` (``models/flashnext/
expert_cache.py:1709-1772``) with every expert resident in HBM, so there is
no expert pool, no SSD read and no host route sync (``:1739-1749``); the
routing stays on the device.  ``MoEBlock`` mirrors the patched
``Qwen3_5MoeSparseMoeBlock.__call__`` = ``_moe_call`` (``adaptive_topk.py:
54-293``) at threshold 1.0 and renorm blend 1.0.
"""
from __future__ import annotations

import torch

from . import ops


class SwitchGLU:
    """Routed experts with a SwiGLU MLP over a resident Q4 bank."""

    metal_combines_scores = True   # the combine is fused into the call

    def __init__(self, weights: ops.MoEWeights):
        self.weights = weights
        self._last_fused_shared = False

    def __call__(self, x, indices, allow_sort=True, scores=None, shared_y=None, shared=None,
                 shared_gate=None):
        """Without ``scores``: per-slot outputs [..., k, d].  With ``scores``:
        the combined [..., d], including ``shared_y`` or ``shared *
        shared_gate`` when given."""
        del allow_sort  # the device path always sorts by expert
        d = self.weights.hidden
        lead = tuple(x.shape[:-1])
        k = int(indices.shape[-1])
        x2 = x.reshape(-1, d)
        r = indices.reshape(-1, k)
        out = ops.moe_experts(x2, r, self.weights,
                              scores=None if scores is None else scores.reshape(-1, k),
                              shared_y=None if shared_y is None else shared_y.reshape(-1, d),
                              shared=None if shared is None else shared.reshape(-1, d),
                              shared_gate=None if shared_gate is None else shared_gate.reshape(-1))
        self._last_fused_shared = scores is not None and (shared_y is not None or shared is not None)
        if scores is None:
            return out.reshape(*lead, k, d)
        return out.reshape(*lead, d)


class MoEBlock:
    """The routed sparse-MoE block: router, top-k, renorm, shared expert,
    routed experts, combine — one device pass."""

    def __init__(self, weights: ops.MoEWeights):
        self.weights = weights
        self.top_k = weights.top_k
        self.switch_mlp = SwitchGLU(weights)

    def gate(self, x):
        """bf16 router logits [..., E]."""
        return ops.router(x, self.weights).logits

    def shared_expert(self, x):
        w = self.weights
        g = ops.quantized_matmul(x, w.shared_gate.weight[0], w.shared_gate.scales[0], w.shared_gate.biases[0])
        u = ops.quantized_matmul(x, w.shared_up.weight[0], w.shared_up.scales[0], w.shared_up.biases[0])
        h = ops.swiglu(g, u)
        return ops.quantized_matmul(h, w.shared_down.weight[0], w.shared_down.scales[0],
                                    w.shared_down.biases[0])

    def shared_expert_gate(self, x):
        w = self.weights.shared_expert_gate
        return ops.quantized_matmul(x, w.weight[0], w.scales[0], w.biases[0])

    def __call__(self, x):
        return ops.moe_block(x, self.weights)


def moe_call(block: MoEBlock, x):
    """``_moe_call(self, x)`` (``adaptive_topk.py:54``)."""
    return block(x)
