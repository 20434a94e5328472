"""Device operators of the MoE hot path, on torch tensors, via libvxmoe.

Every operator runs hand-written sm_100a CUDA through the C ABI on the
current torch stream.  Inputs must be CUDA tensors (bf16 activations,
uint32 packed weights, bf16 scales/biases); nothing here computes on the
CPU and there is no fallback path.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Optional, Sequence

import numpy as np
import torch

from . import _lib
from ._lib import VxMoEWeights, VxQ4

GROUP_SIZE = 32
NATIVE_GROUP = 64   # the one coarser grouping the tiled records keep as stored
BITS = 4


# --------------------------------------------------------------------------
# tensor plumbing
# --------------------------------------------------------------------------


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _require_cuda(t: torch.Tensor, name: str) -> None:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch tensor")
    if not t.is_cuda:
        raise RuntimeError(f"{name} must live on a CUDA device (no CPU path)")


def _bf16(t: torch.Tensor, name: str) -> torch.Tensor:
    _require_cuda(t, name)
    if t.dtype != torch.bfloat16:
        raise TypeError(f"{name} must be bfloat16, got {t.dtype}")
    return t.contiguous()


def _i32(t, device, name: str) -> torch.Tensor:
    if isinstance(t, np.ndarray):
        t = torch.from_numpy(np.ascontiguousarray(t.astype(np.int32)))
    if not isinstance(t, torch.Tensor):
        t = torch.as_tensor(t)
    if t.dtype not in (torch.int32, torch.int64, torch.uint32, torch.int16, torch.uint8):
        raise TypeError(f"{name} must hold integer expert ids, got {t.dtype}")
    if t.dtype == torch.uint32:
        t = t.view(torch.int32)
    return t.to(device=device, dtype=torch.int32).contiguous()


class _Workspace:
    """One growing scratch buffer per (device, stream).  Calls on one stream
    are ordered, so they may share it."""

    def __init__(self):
        self._bufs = {}

    def get(self, nbytes: int, device: torch.device) -> torch.Tensor:
        key = (device.index, torch.cuda.current_stream(device).cuda_stream)
        buf = self._bufs.get(key)
        if buf is None or buf.numel() < nbytes:
            buf = torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)
            self._bufs[key] = buf
        return buf


_WS = _Workspace()


# --------------------------------------------------------------------------
# Q4 projections and MoE weights
# --------------------------------------------------------------------------


@dataclass
class Q4Projection:
    """Packed expert rows of one projection (``Q4G32Projection``,
    ``models/flashnext/metal_runtime.py:39-45``): weight uint32
    [experts, out, in/8], scales/biases bf16 [experts, out, in/group_size].
    group_size is 32, or 64 for a bank kept in its checkpoint grouping
    (``from_group(..., native=True)``), which the kernels read only from a
    tiled pool."""

    weight: torch.Tensor
    scales: torch.Tensor
    biases: torch.Tensor
    group_size: int = GROUP_SIZE

    @property
    def experts(self) -> int:
        return int(self.weight.shape[0])

    @property
    def out_features(self) -> int:
        return int(self.weight.shape[1])

    @property
    def in_features(self) -> int:
        return int(self.weight.shape[2]) * 8

    def validate(self, group_size: Optional[int] = None) -> None:
        group_size = self.group_size if group_size is None else int(group_size)
        w, s, b = self.weight, self.scales, self.biases
        for name, t in (("weight", w), ("scales", s), ("biases", b)):
            _require_cuda(t, name)
            if not t.is_contiguous():
                raise ValueError(f"{name} must be contiguous")
        if w.dtype != torch.uint32:
            raise TypeError("Q4 weights must use uint32 packed values")
        if s.dtype != torch.bfloat16 or b.dtype != torch.bfloat16:
            raise TypeError("Q4 scales and biases must be bfloat16")
        if w.dim() != 3:
            raise ValueError(f"weight shape {tuple(w.shape)} must be [experts, out, in/8]")
        if group_size <= 0 or (w.shape[2] * 8) % group_size:
            raise ValueError(f"{w.shape[2] * 8} inputs do not split into groups of {group_size}")
        meta = (w.shape[0], w.shape[1], w.shape[2] * 8 // group_size)
        if tuple(s.shape) != meta or tuple(b.shape) != meta:
            raise ValueError(f"Q4/G{group_size} scales and biases have an invalid shape")

    def vx(self) -> VxQ4:
        return VxQ4(self.weight.data_ptr(), self.scales.data_ptr(), self.biases.data_ptr(),
                    self.experts, self.out_features, self.in_features, self.group_size)

    @staticmethod
    def from_group(weight: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor,
                   group_size: int, native: bool = False) -> "Q4Projection":
        """A projection quantized in groups of `group_size` (a multiple of
        32, e.g. the G64 checkpoints of models/flashnext/metal_runtime.py:
        950-971).  With `native` a G64 bank is kept as stored (one scale/bias
        pair per 64 inputs; the tiled records carry it that way).  Otherwise
        it takes the kernels' group-32 form: every scale and bias is repeated
        for each 32-input group it covers.  Each dequantized weight
        scale*q + bias is the same either way, and so are the kernels'
        products: their sums run per 32 inputs in both forms."""
        if group_size % GROUP_SIZE or group_size <= 0:
            raise ValueError(f"group size {group_size} is not a multiple of {GROUP_SIZE}")
        if native and group_size == NATIVE_GROUP:
            p = Q4Projection(weight, scales, biases, NATIVE_GROUP)
            p.validate()
            return p
        r = group_size // GROUP_SIZE
        if r > 1:
            scales = scales.repeat_interleave(r, dim=-1).contiguous()
            biases = biases.repeat_interleave(r, dim=-1).contiguous()
        p = Q4Projection(weight, scales, biases)
        p.validate()
        return p

    @staticmethod
    def from_any(value, device=None) -> "Q4Projection":
        """Accept a Q4Projection, a (weight, scales, biases) triple or a
        mapping with those keys; numpy arrays are uploaded (bf16 values held
        in float32 arrays convert exactly)."""
        if isinstance(value, Q4Projection):
            return value
        if isinstance(value, dict):
            value = (value["weight"], value["scales"], value["biases"])
        if hasattr(value, "weight") and hasattr(value, "scales"):
            value = (value.weight, value.scales, value.biases)
        if not isinstance(value, (tuple, list)) or len(value) != 3:
            raise TypeError("projection must be (weight, scales, biases)")
        w, s, b = value
        device = device or torch.device("cuda")
        return Q4Projection(_upload_u32(w, device), _upload_bf16(s, device), _upload_bf16(b, device))


def _upload_u32(w, device) -> torch.Tensor:
    if isinstance(w, np.ndarray):
        if w.dtype != np.uint32:
            raise TypeError("Q4 weights must use uint32 packed values")
        w = torch.from_numpy(np.ascontiguousarray(w))
    if not isinstance(w, torch.Tensor) or w.dtype != torch.uint32:
        raise TypeError("Q4 weights must use uint32 packed values")
    return w.to(device).contiguous()


def _upload_bf16(a, device) -> torch.Tensor:
    if isinstance(a, np.ndarray):
        a = torch.from_numpy(np.ascontiguousarray(a.astype(np.float32)))
    if not isinstance(a, torch.Tensor):
        a = torch.as_tensor(a)
    return a.to(device=device, dtype=torch.bfloat16).contiguous()


class MoEWeights:
    """Resident weights of one routed MoE block: the routed gate/up/down
    banks, the bf16 router, and optionally the shared expert with its gate
    (``adaptive_topk.py:54-293``; checkpoint names ``mlp.switch_mlp.*``,
    ``mlp.gate``, ``mlp.shared_expert.*``, ``mlp.shared_expert_gate``)."""

    def __init__(self, gate, up, down, router_w=None, shared_gate=None, shared_up=None,
                 shared_down=None, shared_expert_gate=None, top_k: int = 10, device=None,
                 check_router: bool = True):
        device = torch.device(device) if device is not None else torch.device("cuda")
        self.gate = Q4Projection.from_any(gate, device)
        self.up = Q4Projection.from_any(up, device)
        self.down = Q4Projection.from_any(down, device)
        self.router_w = None if router_w is None else _upload_bf16(router_w, device)
        has_shared = shared_gate is not None
        self.shared_gate = Q4Projection.from_any(shared_gate, device) if has_shared else None
        self.shared_up = Q4Projection.from_any(shared_up, device) if has_shared else None
        self.shared_down = Q4Projection.from_any(shared_down, device) if has_shared else None
        self.shared_expert_gate = (None if shared_expert_gate is None
                                   else Q4Projection.from_any(shared_expert_gate, device))
        self.top_k = int(top_k)
        self.device = self.gate.weight.device
        for p in self.projections():
            p.validate()
        # routed and shared banks share one grouping: 32, or 64 kept natively
        # (read from the tiled pool only); the shared-expert gate is group 32
        self.group_size = self.gate.group_size
        banks = [p for p in self.projections() if p is not self.shared_expert_gate]
        if any(p.group_size != self.group_size for p in banks):
            raise ValueError("routed and shared banks must share one group size")
        if self.shared_expert_gate is not None and self.shared_expert_gate.group_size != GROUP_SIZE:
            raise ValueError(f"the shared-expert gate takes groups of {GROUP_SIZE}")
        E, I, d = self.num_experts, self.gate.out_features, self.hidden
        if self.up.weight.shape != self.gate.weight.shape:
            raise ValueError("gate and up projection widths must match")
        if tuple(self.down.weight.shape) != (E, d, I // 8):
            raise ValueError(f"down weight shape {tuple(self.down.weight.shape)} != {(E, d, I // 8)}")
        # An expert-parallel shard keeps the full router: check_router=False.
        if check_router and self.router_w is not None and tuple(self.router_w.shape) != (E, d):
            raise ValueError(f"router weight shape {tuple(self.router_w.shape)} != {(E, d)}")
        self.pool: Optional[TiledPool] = None
        # expert pipeline: _lib.PATH_AUTO (GEMV for decode-sized batches,
        # tcgen05 GEMM from four routed positions per expert), PATH_GEMV, PATH_GEMM
        self.expert_path = _lib.PATH_AUTO
        # bf16 [E] added to the bf16 router logits (None: no bias); the
        # skewed-load benchmark puts +2.0 on its hot experts this way
        self.router_bias: Optional[torch.Tensor] = None
        # adaptive top-k, the layer's threshold and minimum keep
        # (adaptive_topk.py set_threshold / set_min_keep, per layer as its
        # _LAYER_THRESHOLDS): below 1.0 a token keeps its leading slots until
        # they hold this share of its top-k probability mass, at least
        # min_keep; 1.0 routes every slot (the exact top-k, the default)
        self.threshold: float = 1.0
        self.min_keep: int = 1
        # partial residency (vxmoe.residency.SlotPool.attach): the slot pool
        # holding this layer's routed records, and the layer's key in it
        self.slot_pool = None
        self.slot_layer = None
        if self.group_size != GROUP_SIZE:
            # native G64 banks are read from the tiled records only
            self.pack()

    def pack(self, down_rows: int = 32) -> "MoEWeights":
        """Re-tile the experts into the resident pool the decode kernels
        stream (one bulk copy per chunk); every later call on these weights
        reads the pool.  A load-time step (the role of the reference's slab
        packing, ``slab_pack.py:1-25``).  Returns self."""
        self.pool = TiledPool(self, down_rows)
        return self

    @property
    def num_experts(self) -> int:
        return self.gate.experts

    @property
    def hidden(self) -> int:
        return self.gate.in_features

    @property
    def intermediate(self) -> int:
        return self.gate.out_features

    def projections(self):
        out = [self.gate, self.up, self.down]
        for p in (self.shared_gate, self.shared_up, self.shared_down, self.shared_expert_gate):
            if p is not None:
                out.append(p)
        return out

    def vx(self, with_shared: bool = True) -> VxMoEWeights:
        s = VxMoEWeights()
        s.gate, s.up, s.down = self.gate.vx(), self.up.vx(), self.down.vx()
        if with_shared and self.shared_gate is not None:
            s.shared_gate, s.shared_up, s.shared_down = (
                self.shared_gate.vx(), self.shared_up.vx(), self.shared_down.vx())
        if self.shared_expert_gate is not None:
            s.shared_expert_gate = self.shared_expert_gate.vx()
        s.router_w = _ptr(self.router_w)
        s.num_experts, s.hidden, s.top_k = self.num_experts, self.hidden, self.top_k
        if self.pool is not None:
            s.pool = ctypes.pointer(self.pool.vx())
        s.expert_path = int(self.expert_path)
        if self.router_bias is not None:   # one value per router row (all experts of the layer)
            n_router = int(self.router_w.shape[0]) if self.router_w is not None else self.num_experts
            s.router_bias = _ptr(_bias(self.router_bias, n_router))
        _set_keep(s, self.threshold, self.min_keep)
        return s

    def nbytes_per_expert(self) -> int:
        return sum(int(t.numel() * t.element_size()) // self.num_experts
                   for p in (self.gate, self.up, self.down)
                   for t in (p.weight, p.scales, p.biases))

    @staticmethod
    def random(num_experts=512, hidden=2048, inter=512, shared_inter=512, top_k=10,
               device=None, generator=None, router_experts=None,
               router_generator=None, group_size: int = GROUP_SIZE) -> "MoEWeights":
        """Synthetic weights with the benchmark distributions: codes uniform
        in 0..15, scale = bf16(|N(0, 0.02)|/8), bias = -8*scale, router
        bf16 N(0, 0.02).  An expert-parallel shard passes the full expert
        count as `router_experts` and a generator shared by all ranks as
        `router_generator` (router and shared expert are replicated).
        group_size 64 makes native G64 banks (packed at construction); the
        shared-expert gate stays group 32."""
        device = torch.device(device) if device is not None else torch.device("cuda")
        g = generator
        gr = router_generator if router_generator is not None else generator
        n_router = router_experts if router_experts is not None else num_experts

        def bank(E, out, inn, gs=group_size):
            w = torch.randint(-2**31, 2**31 - 1, (E, out, inn // 8), dtype=torch.int32,
                              device=device, generator=g).view(torch.uint32)
            s = (torch.randn((E, out, inn // gs), device=device, generator=g).abs()
                 * 0.02 / 8).to(torch.bfloat16)
            b = (s.float() * -8.0).to(torch.bfloat16)
            return Q4Projection(w, s, b, gs)

        gate = bank(num_experts, inter, hidden)
        up = bank(num_experts, inter, hidden)
        down = bank(num_experts, hidden, inter)
        g = gr
        router = (torch.randn((n_router, hidden), device=device, generator=g) * 0.02).to(torch.bfloat16)
        sh = [bank(1, shared_inter, hidden), bank(1, shared_inter, hidden), bank(1, hidden, shared_inter)] \
            if shared_inter else [None, None, None]
        seg = bank(1, 1, hidden, GROUP_SIZE) if shared_inter else None
        return MoEWeights(gate, up, down, router, *sh, seg, top_k=top_k, device=device,
                          check_router=n_router == num_experts)


def tile_bank(a: Q4Projection, b: Optional[Q4Projection] = None, tile_rows: int = 16) -> torch.Tensor:
    """Records of bank `a` (with `b` interleaved as the up half of a gate/up
    pair) in the tiled pool layout, uint8 on a's device."""
    nproj = 1 if b is None else 2
    lib = _lib.load()
    n = lib.vx_q4_tiles_bytes_group(a.experts, a.out_features, a.in_features, nproj, tile_rows,
                                    a.group_size)
    if n == 0:
        raise ValueError(f"no tiled layout for {a.out_features}x{a.in_features}, "
                         f"nproj {nproj}, tile_rows {tile_rows}, group {a.group_size}")
    rec = torch.empty(n, dtype=torch.uint8, device=a.weight.device)
    qa = a.vx()
    qb = b.vx() if b is not None else None
    _lib.check(lib.vx_q4_tile(ctypes.byref(qa), ctypes.byref(qb) if qb is not None else None, nproj,
                              tile_rows, rec.data_ptr(), n, _stream(rec.device)), "tile_bank")
    return rec


class TiledPool:
    """The block's experts re-tiled for the decode GEMV: routed gate/up
    interleaved in 16-row tiles, routed down in `down_rows`-row tiles, and the
    shared expert likewise.  Expert e's records sit at e * stride, the
    counterpart of the reference's fixed-stride slab records
    (``slab_pack.py:1-25``, ``expert_pool.py:1-22``)."""

    def __init__(self, w: "MoEWeights", down_rows: int = 32):
        if down_rows not in (16, 32):
            raise ValueError("down_rows must be 16 or 32")
        self.down_rows = down_rows
        self.group_size = w.group_size
        self.gate_up = tile_bank(w.gate, w.up, 16)
        self.down = tile_bank(w.down, None, down_rows)
        self.shapes = {"gate_up": (w.num_experts, w.intermediate, w.hidden, 2, 16),
                       "down": (w.num_experts, w.hidden, w.intermediate, 1, down_rows)}
        self.shared_gate_up = self.shared_down = None
        if w.shared_gate is not None:
            Is = w.shared_gate.out_features
            self.shared_gate_up = tile_bank(w.shared_gate, w.shared_up, 16)
            self.shared_down = tile_bank(w.shared_down, None, down_rows)
            self.shapes["shared_gate_up"] = (1, Is, w.hidden, 2, 16)
            self.shapes["shared_down"] = (1, w.hidden, Is, 1, down_rows)
        self._struct = _lib.VxMoEPool()
        for name, (E, out, inn, nproj, rows) in self.shapes.items():
            t = getattr(self._struct, name)
            t.records = getattr(self, name).data_ptr()
            t.experts, t.out, t.in_, t.nproj, t.tile_rows = E, out, inn, nproj, rows
            t.group_size = self.group_size
            setattr(self._struct, name, t)

    def vx(self) -> "_lib.VxMoEPool":
        return self._struct

    def nbytes(self) -> int:
        return sum(int(getattr(self, n).numel()) for n in self.shapes)


# --------------------------------------------------------------------------
# operators
# --------------------------------------------------------------------------


def dequantize(w: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor,
               expert: int = 0, group_size: int = GROUP_SIZE) -> torch.Tensor:
    """float32 ``scale*q + bias`` of one expert (``mx.dequantize`` affine,
    ``metal_runtime.py:770-777``); w may be [out, in/8] or [E, out, in/8]."""
    if w.dim() == 2:
        w, scales, biases = w[None], scales[None], biases[None]
    p = Q4Projection(w.contiguous(), scales.contiguous(), biases.contiguous(), int(group_size))
    p.validate()
    out = torch.empty((p.out_features, p.in_features), dtype=torch.float32, device=w.device)
    q = p.vx()
    _lib.check(_lib.load().vx_q4_dequant(ctypes.byref(q), int(expert), out.data_ptr(),
                                          _stream(w.device)), "dequantize")
    return out


def swiglu(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """``silu(gate) * up`` with MLX's bf16 rounding sequence
    (``metal_runtime.py:267-285``)."""
    gate, up = _bf16(gate, "gate"), _bf16(up, "up")
    if gate.shape != up.shape:
        raise ValueError("gate and up must have the same shape")
    out = torch.empty_like(gate)
    _lib.check(_lib.load().vx_swiglu_bf16(gate.data_ptr(), up.data_ptr(), out.data_ptr(),
                                           gate.numel(), _stream(gate.device)), "swiglu")
    return out


def gather_qmm(x, w, scales, biases, lhs_indices=None, rhs_indices=None, transpose=True,
               group_size=GROUP_SIZE, bits=BITS, mode="affine", sorted_indices=False):
    """MLX ``gather_qmm`` for affine Q4 weights (the call at
    ``expert_cache.py:818-829``).

    ``x`` [..., M, K] bf16; ``w`` [E, N, K/8] uint32; scales/biases
    [E, N, K/32] bf16.  ``lhs_indices`` selects x batch entries (default:
    x's own batch positions), ``rhs_indices`` selects experts; both broadcast
    to the output batch shape.  Returns bf16 [*batch, M, N].
    """
    if not transpose:
        raise ValueError("only transpose=True is supported (weights are [E, N, K/8])")
    if bits != BITS or mode != "affine" or group_size != GROUP_SIZE:
        raise ValueError("only affine 4-bit group-32 weights are supported")
    x = _bf16(x, "x")
    proj = Q4Projection(w.contiguous(), scales.contiguous(), biases.contiguous())
    proj.validate(group_size)
    if x.dim() < 2:
        raise ValueError("x must have shape [..., M, K]")
    M, K = int(x.shape[-2]), int(x.shape[-1])
    if K != proj.in_features:
        raise ValueError(f"weight shape {tuple(w.shape)} does not match input width {K}")
    dev = x.device
    xb = tuple(x.shape[:-2])
    nb = int(np.prod(xb)) if xb else 1
    lhs = (torch.arange(nb, device=dev, dtype=torch.int32).reshape(xb) if lhs_indices is None
           else _i32(lhs_indices, dev, "lhs_indices"))
    if rhs_indices is None:
        raise ValueError("rhs_indices is required")
    host_rhs = rhs_indices if isinstance(rhs_indices, np.ndarray) else None
    rhs = _i32(rhs_indices, dev, "rhs_indices")
    if host_rhs is not None and host_rhs.size and (host_rhs.min() < 0 or host_rhs.max() >= proj.experts):
        raise ValueError("rhs_indices contain an expert outside the bank")
    shape = torch.broadcast_shapes(tuple(lhs.shape), tuple(rhs.shape))
    lhs_b = lhs.expand(shape).reshape(-1).contiguous()
    rhs_b = rhs.expand(shape).reshape(-1).contiguous()
    B = int(lhs_b.numel())
    N = proj.out_features
    out = torch.zeros((*shape, M, N), dtype=torch.bfloat16, device=dev)
    if B == 0:
        return out
    lib = _lib.load()
    nbytes = lib.vx_gather_qmm_workspace(B, M, proj.experts, nb * M, K)
    ws = _WS.get(nbytes, dev)
    q = proj.vx()
    _lib.check(lib.vx_gather_qmm(x.data_ptr(), nb * M, ctypes.byref(q), lhs_b.data_ptr(),
                                 rhs_b.data_ptr(), B, M, int(bool(sorted_indices)),
                                 out.data_ptr(), ws.data_ptr(), ws.numel(), _stream(dev)),
               "gather_qmm")
    return out


def quantized_matmul(x, w, scales, biases, transpose=True, group_size=GROUP_SIZE, bits=BITS):
    """Dense Q4 ``x @ dequant(w).T`` (MLX ``quantized_matmul``) for a
    single projection w [N, K/8]: a one-expert gather_qmm."""
    lead = x.shape[:-1]
    x2 = x.reshape(-1, 1, x.shape[-1])
    idx = torch.zeros((x2.shape[0],), dtype=torch.int32, device=x.device)
    out = gather_qmm(x2, w[None] if w.dim() == 2 else w,
                     scales[None] if scales.dim() == 2 else scales,
                     biases[None] if biases.dim() == 2 else biases,
                     rhs_indices=idx, transpose=transpose, group_size=group_size, bits=bits)
    return out.reshape(*lead, out.shape[-1])


@dataclass
class TopK:
    inds: torch.Tensor      # int32 [T, k]
    weights: torch.Tensor   # bf16 [T, k] renormalised
    scores: torch.Tensor    # bf16 [T, k] selected probabilities
    mass: torch.Tensor      # bf16 [T]


def softmax_topk(logits: torch.Tensor, k: int) -> TopK:
    """``softmax(precise) -> top-k -> scores -> mass -> renorm`` over bf16
    logits (``adaptive_topk.py:59-65``, ``:257-262``)."""
    logits = _bf16(logits, "logits")
    lead = logits.shape[:-1]
    E = int(logits.shape[-1])
    l2 = logits.reshape(-1, E)
    T = int(l2.shape[0])
    dev = logits.device
    inds = torch.empty((T, k), dtype=torch.int32, device=dev)
    weights = torch.empty((T, k), dtype=torch.bfloat16, device=dev)
    scores = torch.empty((T, k), dtype=torch.bfloat16, device=dev)
    mass = torch.empty((T,), dtype=torch.bfloat16, device=dev)
    _lib.check(_lib.load().vx_softmax_topk(l2.data_ptr(), T, E, int(k), inds.data_ptr(),
                                            scores.data_ptr(), weights.data_ptr(), mass.data_ptr(),
                                            _stream(dev)), "softmax_topk")
    return TopK(inds.reshape(*lead, k), weights.reshape(*lead, k), scores.reshape(*lead, k),
                mass.reshape(*lead))


@dataclass
class RouterOut:
    logits: torch.Tensor
    inds: torch.Tensor
    weights: torch.Tensor
    shared_gate: Optional[torch.Tensor]


def router(x: torch.Tensor, weights: MoEWeights) -> RouterOut:
    """Router of the block: bf16 logits, top-k, renormalised weights and the
    shared expert's sigmoid gate."""
    return route(x, weights.router_w, weights.top_k, weights.shared_expert_gate,
                 router_bias=weights.router_bias, threshold=weights.threshold,
                 min_keep=weights.min_keep)


def _set_keep(s: VxMoEWeights, threshold: float, min_keep: int) -> None:
    """Adaptive top-k settings of a weights struct: keep_mass 0 routes every
    slot (threshold 1.0 or more, the reference's exact path)."""
    t = float(threshold)
    if not (t > 0.0):
        raise ValueError(f"routing threshold must be positive, got {threshold}")
    s.keep_mass = t if t < 1.0 else 0.0
    s.keep_min = max(1, int(min_keep))


def _bias(b: torch.Tensor, E: int) -> torch.Tensor:
    """The bias tensor itself (its pointer goes to the library, so no copy)."""
    _require_cuda(b, "router_bias")
    if b.dtype != torch.bfloat16:
        raise TypeError(f"router_bias must be bfloat16, got {b.dtype}")
    if b.numel() != E or not b.is_contiguous():
        raise ValueError(f"router_bias must be a contiguous vector of {E} values")
    return b


def route(x: torch.Tensor, router_w: torch.Tensor, top_k: int,
          shared_expert_gate: Optional[Q4Projection] = None,
          router_bias: Optional[torch.Tensor] = None, threshold: float = 1.0,
          min_keep: int = 1) -> RouterOut:
    """The router from its own tensors: bf16 gate [E, d] and, optionally,
    the Q4 shared-expert gate [1, 1, d/8] and a bf16 logit bias [E] (no
    expert bank needed).  threshold < 1.0: adaptive top-k (a token's slots
    past its keep count name its first expert with weight 0)."""
    x = _bf16(x, "x")
    router_w = _bf16(router_w, "router_w")
    E, d = int(router_w.shape[0]), int(router_w.shape[1])
    x2 = x.reshape(-1, d)
    T = int(x2.shape[0])
    dev = x.device
    k = int(top_k)
    logits = torch.empty((T, E), dtype=torch.bfloat16, device=dev)
    inds = torch.empty((T, k), dtype=torch.int32, device=dev)
    w = torch.empty((T, k), dtype=torch.bfloat16, device=dev)
    sg = torch.empty((T,), dtype=torch.bfloat16, device=dev) if shared_expert_gate is not None else None
    st = VxMoEWeights()
    st.router_w = router_w.data_ptr()
    if shared_expert_gate is not None:
        st.shared_expert_gate = shared_expert_gate.vx()
    st.num_experts, st.hidden, st.top_k = E, d, k
    if router_bias is not None:
        st.router_bias = _ptr(_bias(router_bias, E))
    _set_keep(st, threshold, min_keep)
    lib = _lib.load()
    ws = _WS.get(lib.vx_router_workspace(T, ctypes.byref(st)), dev)
    _lib.check(lib.vx_router(x2.data_ptr(), T, ctypes.byref(st), logits.data_ptr(),
                             inds.data_ptr(), w.data_ptr(), _ptr(sg), ws.data_ptr(), ws.numel(),
                             _stream(dev)), "router")
    lead = x.shape[:-1]
    return RouterOut(logits.reshape(*lead, E), inds.reshape(*lead, k), w.reshape(*lead, k),
                     None if sg is None else sg.reshape(*lead, 1))


@dataclass
class Permutation:
    order: torch.Tensor     # int32 [P]  flat index at each sorted position
    inverse: torch.Tensor   # int32 [P]  sorted position of each flat index
    offsets: torch.Tensor   # int32 [E+1]
    errors: torch.Tensor    # int32 [1]  ids outside [0, E)


def permute(ids: torch.Tensor, num_experts: int) -> Permutation:
    """Stable sort of flat expert ids (mlx-vlm ``_gather_sort``)."""
    _require_cuda(ids, "ids")
    ids = _i32(ids, ids.device, "ids").reshape(-1)
    dev = ids.device
    P = int(ids.numel())
    order = torch.empty((P,), dtype=torch.int32, device=dev)
    inverse = torch.empty((P,), dtype=torch.int32, device=dev)
    offsets = torch.empty((num_experts + 1,), dtype=torch.int32, device=dev)
    errors = torch.zeros((1,), dtype=torch.int32, device=dev)
    lib = _lib.load()
    ws = _WS.get(lib.vx_permute_workspace(P, num_experts), dev)
    _lib.check(lib.vx_permute(ids.data_ptr(), P, int(num_experts), order.data_ptr(),
                              inverse.data_ptr(), offsets.data_ptr(), errors.data_ptr(),
                              ws.data_ptr(), ws.numel(), _stream(dev)), "permute")
    return Permutation(order, inverse, offsets, errors)


def moe_experts(x: torch.Tensor, routes, weights: MoEWeights, scores=None, shared_y=None,
                shared=None, shared_gate=None, path: Optional[int] = None) -> torch.Tensor:
    """Routed experts for given routes (the executor contract,
    ``metal_runtime.py:799-974``).  With ``scores`` returns [T, d]: the
    float32 score-weighted combine of bf16 slot outputs plus the shared part;
    without, returns the per-slot outputs [T, k, d].  ``path`` overrides the
    weights' expert pipeline for this call (``_lib.PATH_*``)."""
    x = _bf16(x, "x")
    d = weights.hidden
    x2 = x.reshape(-1, d)
    T = int(x2.shape[0])
    dev = x.device
    r = _i32(routes, dev, "routes").reshape(T, -1)
    k = int(r.shape[1])
    if shared is not None and shared_gate is None or shared is None and shared_gate is not None:
        raise ValueError("shared and shared_gate must be provided together")
    if shared_y is not None and shared is not None:
        raise ValueError("provide shared_y or shared parts, not both")
    sc = None if scores is None else _bf16(scores.to(torch.bfloat16) if scores.dtype != torch.bfloat16 else scores, "scores").reshape(T, k)
    sy = None if shared_y is None else _bf16(shared_y.to(torch.bfloat16), "shared_y").reshape(T, d)
    sh = None if shared is None else _bf16(shared.to(torch.bfloat16), "shared").reshape(T, d)
    shg = None if shared_gate is None else _bf16(shared_gate.to(torch.bfloat16), "shared_gate").reshape(T)
    if weights.slot_pool is not None:   # partially resident: fill the routes' misses
        weights.slot_pool.ensure(weights, [e for e in torch.unique(r).tolist() if 0 <= e < weights.num_experts])
    st = weights.vx(with_shared=False)
    st.top_k = k
    if path is not None:
        st.expert_path = int(path)
    lib = _lib.load()
    ws = _WS.get(lib.vx_moe_experts_workspace(T, ctypes.byref(st)), dev)
    out = torch.empty((T, d) if sc is not None else (T, k, d), dtype=torch.bfloat16, device=dev)
    _lib.check(lib.vx_moe_experts(x2.data_ptr(), T, r.data_ptr(), _ptr(sc), ctypes.byref(st),
                                  _ptr(sy), _ptr(sh), _ptr(shg), out.data_ptr(), ws.data_ptr(),
                                  ws.numel(), _stream(dev)), "moe_experts")
    return out


def moe_experts_partial(x: torch.Tensor, routes: torch.Tensor, scores: torch.Tensor,
                        weights: MoEWeights) -> torch.Tensor:
    """Expert-parallel share: float32 [T, d] unrounded slot-order sum of
    bf16(y_s)*score_s over the slots whose route is an expert of this bank
    (routes -1 elsewhere)."""
    x = _bf16(x, "x")
    d = weights.hidden
    x2 = x.reshape(-1, d)
    T = int(x2.shape[0])
    dev = x.device
    r = _i32(routes, dev, "routes").reshape(T, -1)
    k = int(r.shape[1])
    sc = _bf16(scores, "scores").reshape(T, k)
    st = weights.vx(with_shared=False)
    st.top_k = k
    lib = _lib.load()
    out = torch.empty((T, d), dtype=torch.float32, device=dev)
    if T == 0:
        return out
    ws = _WS.get(lib.vx_moe_experts_workspace(T, ctypes.byref(st)), dev)
    _lib.check(lib.vx_moe_experts_partial(x2.data_ptr(), T, r.data_ptr(), sc.data_ptr(),
                                          ctypes.byref(st), out.data_ptr(), ws.data_ptr(),
                                          ws.numel(), _stream(dev)), "moe_experts_partial")
    return out


def moe_block(x: torch.Tensor, weights: MoEWeights, return_routing: bool = False):
    """The whole routed MoE block at threshold 1.0 (``_moe_call``,
    ``adaptive_topk.py:54-293``): y [..., d] bf16."""
    x = _bf16(x, "x")
    d = weights.hidden
    if weights.router_w is None:
        raise ValueError("the block needs the router weight")
    x2 = x.reshape(-1, d)
    T = int(x2.shape[0])
    dev = x.device
    k = weights.top_k
    if weights.slot_pool is not None:   # partially resident: route, then fill the misses
        r = router(x2, weights)
        weights.slot_pool.ensure(weights, torch.unique(r.inds).tolist())
    st = weights.vx()
    lib = _lib.load()
    ws = _WS.get(lib.vx_moe_block_workspace(T, ctypes.byref(st)), dev)
    y = torch.empty((T, d), dtype=torch.bfloat16, device=dev)
    inds = torch.empty((T, k), dtype=torch.int32, device=dev) if return_routing else None
    w = torch.empty((T, k), dtype=torch.bfloat16, device=dev) if return_routing else None
    _lib.check(lib.vx_moe_block(x2.data_ptr(), T, ctypes.byref(st), y.data_ptr(), _ptr(inds),
                                _ptr(w), ws.data_ptr(), ws.numel(), _stream(dev)), "moe_block")
    y = y.reshape(*x.shape[:-1], d)
    if return_routing:
        return y, inds.reshape(*x.shape[:-1], k), w.reshape(*x.shape[:-1], k)
    return y


class GraphedBlock:
    """``moe_block`` for a fixed batch size captured once into a CUDA graph:
    a call copies x into the graph's input buffer and replays the block
    (router through combine, every launch of it) as one graph launch.  The
    library's entry points never synchronise the host or allocate, so the
    whole block captures; the output tensor belongs to the graph and is
    overwritten by the next call."""

    def __init__(self, weights: MoEWeights, tokens: int):
        dev = weights.device
        self.weights = weights
        self.x = torch.zeros((int(tokens), weights.hidden), dtype=torch.bfloat16, device=dev)
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            moe_block(self.x, weights)            # kernel attributes, workspace
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize(dev)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.y = moe_block(self.x, weights)

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        self.x.copy_(x, non_blocking=True)
        self.graph.replay()
        return self.y


def rms_norm(x: torch.Tensor, gain: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """float32 RMSNorm with gain, bf16 out (``patch_rmsnorm.py:96-120``)."""
    x = _bf16(x, "x")
    gain = _bf16(gain, "gain")
    d = int(x.shape[-1])
    if gain.numel() != d:
        raise ValueError("gain must have the hidden size")
    x2 = x.reshape(-1, d)
    y = torch.empty_like(x2)
    _lib.check(_lib.load().vx_rmsnorm(x2.data_ptr(), gain.data_ptr(), int(x2.shape[0]), d,
                                       float(eps), y.data_ptr(), _stream(x.device)), "rms_norm")
    return y.reshape(x.shape)
