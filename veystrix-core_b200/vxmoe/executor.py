"""The MoE executor surface of the reference, on B200.

Mirrors ``MetalMoEExecutor`` (``models/flashnext/metal_runtime.py:427-983``):
the constructor bounds, ``execute(x, routes, projections, *, scores=...,
shared_y=..., shared=..., shared_gate=..., return_all=...)``, the
combine-only call forms, ``available``/``last_path`` and the error types.
Unlike the reference there is no reference (CPU/MLX) fallback: when the CUDA
library or device is unavailable ``execute`` raises ``RuntimeError``.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Mapping, Sequence

import numpy as np
import torch

from . import ops

MAX_EXPERTS = 1024
MAX_TOP_K = 16
MAX_WIDTH = 16_384
MAX_TOKENS = 1 << 20
GROUP_SIZE = 32
SUPPORTED_GROUP_SIZES = (32,)
BITS = 4
NATIVE_PATH = "custom-cuda"

Q4G32Projection = ops.Q4Projection


@dataclass(frozen=True)
class Capabilities:
    """Backend probe result (``MetalCapabilities``, ``metal_runtime.py:48-62``)."""

    available: bool
    supports_custom_moe: bool
    backend: str
    reason: str

    def __getitem__(self, key: str) -> Any:
        return getattr(self, key)


def probe_capabilities(backend: Any = None) -> Capabilities:
    """Report whether the CUDA library and an sm_100 device are usable,
    without launching a kernel.  ``backend`` may be an injected object with
    ``available``/``supports_custom_moe`` attributes (for tests)."""
    if backend is not None and hasattr(backend, "available"):
        available = bool(getattr(backend, "available"))
        supports = bool(getattr(backend, "supports_custom_moe", False))
        return Capabilities(available and supports, supports, "injected",
                            "injected backend capability")
    if backend not in (None, "cuda"):
        return Capabilities(False, False, str(backend), "unknown backend")
    try:
        from . import _lib
        _lib.load()
    except Exception as exc:  # library missing
        return Capabilities(False, False, "cuda", f"libvxmoe unavailable: {exc}")
    if not torch.cuda.is_available():
        return Capabilities(False, False, "cuda", "no CUDA device")
    major, minor = torch.cuda.get_device_capability()
    if major != 10:
        return Capabilities(False, False, "cuda", f"needs sm_100 (found sm_{major}{minor})")
    return Capabilities(True, True, "cuda", "B200 device detected")


def weighted_combine(expert_outputs, routes, scores):
    """``sum(selected * scores[..., None], axis=-2)`` where ``selected`` is
    the slot form or, when outputs hold every expert, the routed experts
    (``metal_runtime.py:145-191``).  CUDA tensors (bf16 or float32) run the
    library's combine kernel (vx_weighted_combine); host arrays are combined
    on the host, as the reference helper does for NumPy arrays."""
    if isinstance(expert_outputs, torch.Tensor) and expert_outputs.is_cuda:
        return _weighted_combine_cuda(expert_outputs, routes, scores)
    if isinstance(expert_outputs, np.ndarray):
        out, r, s = expert_outputs, np.asarray(routes), np.asarray(scores)
        take = lambda a, i: np.take_along_axis(a, i[..., None], axis=-2)
    else:
        out = expert_outputs
        r = routes if isinstance(routes, torch.Tensor) else torch.as_tensor(np.asarray(routes))
        s = scores if isinstance(scores, torch.Tensor) else torch.as_tensor(np.asarray(scores))
        r = r.to(out.device)
        s = s.to(out.device)
        take = lambda a, i: torch.take_along_dim(a, i[..., None].long(), dim=-2)
    oshape, rshape, sshape = tuple(out.shape), tuple(r.shape), tuple(s.shape)
    if len(oshape) < 2 or len(rshape) == 0:
        raise ValueError("expert_outputs and routes need at least one dimension")
    if sshape != rshape:
        raise ValueError("routes and scores must have identical shapes")
    if oshape[:-1] == rshape:
        sel = out
    elif len(oshape) == len(rshape) + 1 and oshape[-2] >= rshape[-1]:
        count = r.numel() if isinstance(r, torch.Tensor) else r.size
        if count and (int(r.min()) < 0 or int(r.max()) >= oshape[-2]):
            raise ValueError("routes contain an expert outside expert_outputs")
        sel = take(out, r)
    else:
        raise ValueError(f"expert_outputs shape {oshape} does not match routes {rshape}")
    return (sel * s[..., None]).sum(-2)


def _weighted_combine_cuda(out: torch.Tensor, routes, scores) -> torch.Tensor:
    from . import _lib
    dev = out.device
    r = routes if isinstance(routes, torch.Tensor) else torch.as_tensor(np.asarray(routes))
    s = scores if isinstance(scores, torch.Tensor) else torch.as_tensor(np.asarray(scores))
    oshape, rshape, sshape = tuple(out.shape), tuple(r.shape), tuple(s.shape)
    if len(oshape) < 2 or len(rshape) == 0:
        raise ValueError("expert_outputs and routes need at least one dimension")
    if sshape != rshape:
        raise ValueError("routes and scores must have identical shapes")
    if out.dtype not in (torch.bfloat16, torch.float32):
        raise TypeError(f"expert_outputs must be bfloat16 or float32, got {out.dtype}")
    k, d = int(rshape[-1]), int(oshape[-1])
    lead = rshape[:-1]
    T = int(np.prod(lead)) if lead else 1
    if oshape[:-1] == rshape:
        n_out, r_dev = k, None
    elif len(oshape) == len(rshape) + 1 and oshape[:-2] == lead and oshape[-2] >= k:
        n_out = int(oshape[-2])
        r_dev = r.to(device=dev, dtype=torch.int32).reshape(T, k).contiguous()
        if r_dev.numel() and (int(r_dev.min()) < 0 or int(r_dev.max()) >= n_out):
            raise ValueError("routes contain an expert outside expert_outputs")
    else:
        raise ValueError(f"expert_outputs shape {oshape} does not match routes {rshape}")
    o = out.reshape(T, n_out, d).contiguous()
    sc = s.to(device=dev, dtype=out.dtype).reshape(T, k).contiguous()
    y = torch.empty((T, d), dtype=out.dtype, device=dev)
    dtype = _lib.VX_DTYPE_BF16 if out.dtype == torch.bfloat16 else _lib.VX_DTYPE_F32
    stream = torch.cuda.current_stream(dev).cuda_stream
    _lib.check(_lib.load().vx_weighted_combine(o.data_ptr(), dtype, n_out,
                                               None if r_dev is None else r_dev.data_ptr(),
                                               sc.data_ptr(), T, k, d, y.data_ptr(), None, stream),
               "weighted_combine")
    return y.reshape(*lead, d)


def _as_projection(value, device) -> ops.Q4Projection:
    return ops.Q4Projection.from_any(value, device)


class MoEExecutor:
    """Three-projection routed-expert executor on hand-written sm_100a CUDA."""

    def __init__(self, expert_count: int, hidden_size: int, top_k: int, backend: Any = None, *,
                 max_tokens: int = MAX_TOKENS, max_width: int = MAX_WIDTH,
                 group_size: int = GROUP_SIZE, device=None, **_ignored) -> None:
        if not 1 <= expert_count <= MAX_EXPERTS:
            raise ValueError(f"expert_count must be in 1..{MAX_EXPERTS}")
        if hidden_size <= 0:
            raise ValueError("hidden_size must be positive")
        if not 1 <= top_k <= MAX_TOP_K:
            raise ValueError(f"top_k must be in 1..{MAX_TOP_K}")
        if top_k > expert_count:
            raise ValueError("top_k cannot exceed expert_count")
        if not 1 <= max_tokens <= MAX_TOKENS:
            raise ValueError(f"max_tokens must be in 1..{MAX_TOKENS}")
        if not 1 <= max_width <= MAX_WIDTH:
            raise ValueError(f"max_width must be in 1..{MAX_WIDTH}")
        if group_size not in SUPPORTED_GROUP_SIZES:
            raise ValueError(f"group_size must be one of {SUPPORTED_GROUP_SIZES}")
        self.expert_count = int(expert_count)
        self.hidden_size = int(hidden_size)
        self.top_k = int(top_k)
        self.max_tokens = int(max_tokens)
        self.max_width = int(max_width)
        self.group_size = int(group_size)
        self.backend = backend
        self.capabilities = probe_capabilities(backend)
        self.device = torch.device(device) if device is not None else None
        self.last_path = None
        self.fallback_reason = None if self.available else self.capabilities.reason
        self._weights_cache: dict = {}

    @property
    def available(self) -> bool:
        return bool(self.capabilities["available"])

    def _require(self):
        if not self.capabilities.supports_custom_moe or not self.available:
            raise RuntimeError(f"custom MoE is unavailable on this backend ({self.capabilities.reason})")

    def _dev(self, x):
        if isinstance(x, torch.Tensor) and x.is_cuda:
            return x.device
        return self.device or torch.device("cuda")

    def _weights(self, projections, device) -> ops.MoEWeights:
        key = id(projections)
        hit = self._weights_cache.get(key)
        if hit is not None and hit[0] is projections:
            return hit[1]
        if isinstance(projections, Mapping):
            gate, up, down = (projections[n] for n in ("gate_proj", "up_proj", "down_proj"))
        else:
            if len(projections) != 3:
                raise ValueError("projections must contain gate, up, and down")
            gate, up, down = projections
        gate, up, down = (_as_projection(p, device) for p in (gate, up, down))
        gw, iw = gate.out_features, up.out_features
        if gw != iw or gw > self.max_width:
            raise ValueError("gate and up projection widths must match the bound")
        for name, p, inw, outw in (("gate", gate, self.hidden_size, gw),
                                   ("up", up, self.hidden_size, iw),
                                   ("down", down, iw, self.hidden_size)):
            exp = (p.experts, outw, inw // 8)
            if tuple(p.weight.shape) != exp:
                raise ValueError(f"weight shape {tuple(p.weight.shape)} != {exp}")
            p.validate(self.group_size)
        if self.hidden_size % self.group_size or iw % self.group_size:
            raise ValueError(f"Q4/G{self.group_size} projection inputs must be group aligned")
        w = ops.MoEWeights(gate, up, down, top_k=self.top_k, device=device)
        self._weights_cache = {key: (projections, w)}
        return w

    def execute(self, x: Any, routes: Any, projections: Any = None, *, return_all: bool = False,
                scores: Any = None, shared_y: Any = None, shared: Any = None,
                shared_gate: Any = None, **_ignored) -> Any:
        """Run gate, up, SwiGLU and down for flattened inputs.

        ``x`` [tokens, hidden] bf16, ``routes`` [tokens, top_k] expert ids.
        With ``scores`` the result is the combined [tokens, hidden];
        without, one output per slot [tokens, top_k, hidden].  Combine-only
        forms (``execute(outputs, routes, scores)``) weight already
        projected values.
        """
        if projections is not None and not isinstance(projections, (Mapping, list, tuple)):
            self._require()
            self.last_path, self.fallback_reason = NATIVE_PATH, None
            return weighted_combine(x, routes, projections)
        if projections is None and scores is not None:
            self._require()
            self.last_path, self.fallback_reason = NATIVE_PATH, None
            return weighted_combine(x, routes, scores)
        if projections is None:
            raise TypeError("packed execution needs gate, up, and down projections")
        x_shape = tuple(x.shape)
        r_shape = tuple(routes.shape)
        if len(x_shape) != 2 or x_shape[1] != self.hidden_size:
            raise ValueError("x must have shape (tokens, hidden_size)")
        if len(r_shape) != 2 or r_shape[1] != self.top_k:
            raise ValueError("routes must have shape (tokens, top_k)")
        if scores is not None and tuple(scores.shape) != r_shape:
            raise ValueError("scores must have the same shape as routes")
        if (shared is None) != (shared_gate is None):
            raise ValueError("shared and shared_gate must be provided together")
        if shared_y is not None and shared is not None:
            raise ValueError("provide shared_y or shared parts, not both")
        tokens = x_shape[0]
        if r_shape[0] != tokens:
            raise ValueError("x and routes must have the same token count")
        if not 1 <= tokens <= self.max_tokens:
            raise ValueError(f"tokens must be in 1..{self.max_tokens}")
        if isinstance(routes, np.ndarray) and routes.size and (
                routes.min() < 0 or routes.max() >= self.expert_count):
            raise ValueError("routes contain an expert outside the configured bank")
        self._require()
        dev = self._dev(x)
        w = self._weights(projections, dev)
        xt = self._tensor_bf16(x, dev)
        rt = ops._i32(routes, dev, "routes")
        if return_all:
            g = ops.gather_qmm(xt[:, None, None, :], w.gate.weight, w.gate.scales, w.gate.biases,
                               rhs_indices=rt).squeeze(-2)
            u = ops.gather_qmm(xt[:, None, None, :], w.up.weight, w.up.scales, w.up.biases,
                               rhs_indices=rt).squeeze(-2)
            h = ops.swiglu(g, u)
            dn = ops.gather_qmm(h[:, :, None, :], w.down.weight, w.down.scales, w.down.biases,
                                rhs_indices=rt).squeeze(-2)
            self.last_path, self.fallback_reason = NATIVE_PATH, None
            return g, u, dn
        sc = None if scores is None else self._tensor_bf16(scores, dev)
        sy = None if shared_y is None else self._tensor_bf16(shared_y, dev)
        sh = None if shared is None else self._tensor_bf16(shared, dev)
        shg = None if shared_gate is None else self._tensor_bf16(shared_gate, dev)
        out = ops.moe_experts(xt, rt, w, scores=sc, shared_y=sy, shared=sh, shared_gate=shg)
        self.last_path, self.fallback_reason = NATIVE_PATH, None
        return out

    @staticmethod
    def _tensor_bf16(v, dev):
        if isinstance(v, np.ndarray):
            v = torch.from_numpy(np.ascontiguousarray(v.astype(np.float32)))
        if not isinstance(v, torch.Tensor):
            v = torch.as_tensor(v)
        return v.to(device=dev, dtype=torch.bfloat16).contiguous()


def build_executor(expert_count=None, hidden_size=None, top_k=None, packs=None, projections=None,
                   group_size=GROUP_SIZE, bits=BITS, mode="affine", backend=None, **kwargs):
    """Builder entry point (the name ``bench_runtime_layer._load_target``
    looks for first, ``tests/bench/bench_runtime_layer.py:85-100``)."""
    if bits != BITS or mode != "affine":
        raise ValueError("only affine 4-bit weights are supported")
    packs = packs if packs is not None else projections
    if expert_count is None and packs is not None:
        first = packs["gate_proj"] if isinstance(packs, Mapping) else packs[0]
        expert_count = int(first[0].shape[0])
    if hidden_size is None and packs is not None:
        down = packs["down_proj"] if isinstance(packs, Mapping) else packs[2]
        hidden_size = int(down[0].shape[1])
    if top_k is None:
        top_k = min(10, int(expert_count))
    return MoEExecutor(int(expert_count), int(hidden_size), int(top_k), backend,
                       group_size=group_size, **kwargs)


create_executor = build_executor
Executor = MoEExecutor
