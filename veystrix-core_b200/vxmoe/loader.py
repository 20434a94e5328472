"""Loading a routed MoE layer from a safetensors checkpoint.

The checkpoint layout is the one the reference's Flash-Next loader reads
(models/flashnext/loader.py:356-376, preflight.py:68-75): per decoder layer
``language_model.model.layers.{i}.mlp.`` followed by

* ``switch_mlp.{gate,up,down}_proj.{weight,scales,biases}`` - the routed
  experts, uint32-packed 4-bit codes with bf16 scales and biases,
* ``shared_expert.{gate,up,down}_proj.{weight,scales,biases}`` - the shared
  expert, the same format with one expert,
* ``shared_expert_gate.{weight,scales,biases}`` - its quantized sigmoid gate,
* ``gate.weight`` - the router, bf16, unquantized.

The quantization of each layer is inferred from its tensor shapes, as the
reference does per layer (``infer_switch_quantization``, loader.py:379-401),
because converted checkpoints may mix layouts.  The kernels take 4-bit codes
in groups of 32, or of 64 kept as stored in the tiled records; other
multiples of 32 (128, ...) are expanded to groups of 32 at load time
(Q4Projection.from_group), other layouts are rejected with ValueError.

The reader is a small safetensors parser (8-byte little-endian header length,
a JSON header, then the raw tensors); tensors are memory-mapped and copied to
the device one at a time.
"""
from __future__ import annotations

import json
import os
import struct
from dataclasses import dataclass
from typing import Dict, Iterable, List, Optional, Sequence, Tuple

import numpy as np
import torch

from . import ops

HEADER_LIMIT = 100 * 1024 * 1024   # the reference's own bound for a safetensors header

# safetensors dtype -> (numpy storage dtype, torch dtype of the device tensor)
_DTYPES = {
    "U32": (np.uint32, torch.uint32),
    "I32": (np.int32, torch.int32),
    "BF16": (np.uint16, torch.bfloat16),   # bit patterns, viewed as bf16 on the device
    "F16": (np.float16, torch.float16),
    "F32": (np.float32, torch.float32),
    "U8": (np.uint8, torch.uint8),
}


@dataclass
class TensorRef:
    file: str
    dtype: str
    shape: Tuple[int, ...]
    begin: int            # absolute byte offset in the file
    end: int


class SafeTensorStore:
    """The tensors of one or more .safetensors files, by name."""

    def __init__(self, paths: Iterable[str]):
        self.refs: Dict[str, TensorRef] = {}
        for path in paths:
            self._index(path)

    @classmethod
    def from_dir(cls, directory: str) -> "SafeTensorStore":
        names = sorted(n for n in os.listdir(directory) if n.endswith(".safetensors"))
        if not names:
            raise FileNotFoundError(f"no .safetensors files in {directory}")
        return cls(os.path.join(directory, n) for n in names)

    def _index(self, path: str) -> None:
        with open(path, "rb") as fh:
            head = fh.read(8)
            if len(head) != 8:
                raise ValueError(f"{path}: truncated safetensors header")
            (n,) = struct.unpack("<Q", head)
            if n <= 0 or n > HEADER_LIMIT:
                raise ValueError(f"{path}: header length {n} out of range")
            header = json.loads(fh.read(n))
        size = os.path.getsize(path)
        base = 8 + n
        for name, spec in header.items():
            if name == "__metadata__":
                continue
            dtype = spec["dtype"]
            if dtype not in _DTYPES:
                raise ValueError(f"{path}: tensor {name} has unsupported dtype {dtype}")
            begin, end = (int(v) for v in spec["data_offsets"])
            shape = tuple(int(v) for v in spec["shape"])
            count = int(np.prod(shape)) if shape else 1
            if end - begin != count * np.dtype(_DTYPES[dtype][0]).itemsize or base + end > size:
                raise ValueError(f"{path}: tensor {name} has inconsistent offsets")
            self.refs[name] = TensorRef(path, dtype, shape, base + begin, base + end)

    def __contains__(self, name: str) -> bool:
        return name in self.refs

    def shape(self, name: str) -> Tuple[int, ...]:
        return self.refs[name].shape

    def numpy(self, name: str) -> np.ndarray:
        ref = self.refs[name]
        np_dtype = _DTYPES[ref.dtype][0]
        count = int(np.prod(ref.shape)) if ref.shape else 1
        mm = np.memmap(ref.file, dtype=np_dtype, mode="r", offset=ref.begin, shape=(count,))
        return np.asarray(mm).reshape(ref.shape)

    def tensor(self, name: str, device) -> torch.Tensor:
        ref = self.refs[name]
        host = torch.from_numpy(np.array(self.numpy(name), copy=True))   # writable host copy
        torch_dtype = _DTYPES[ref.dtype][1]
        if ref.dtype == "BF16":
            host = host.view(torch.bfloat16)
        elif ref.dtype == "U32":
            host = host.view(torch.int32).view(torch.uint32)
        else:
            host = host.to(torch_dtype)
        return host.to(device)


def infer_switch_quantization(store: SafeTensorStore, prefix: str) -> Tuple[int, int]:
    """(group_size, bits) of one expert block from its tensor shapes: the
    down projection's middle dimension is the hidden width the gate/up
    projections read; bits follow from the packed gate width, the group size
    from the gate's scale count (loader.py:379-401)."""
    packed = int(store.shape(f"{prefix}.gate_proj.weight")[-1])
    groups = int(store.shape(f"{prefix}.gate_proj.scales")[-1])
    hidden = int(store.shape(f"{prefix}.down_proj.weight")[1])
    if packed <= 0 or groups <= 0 or hidden <= 0:
        raise ValueError(f"invalid switch quantization shapes at {prefix}")
    if (packed * 32) % hidden or hidden % groups:
        raise ValueError(f"incompatible switch quantization shapes at {prefix}")
    return hidden // groups, packed * 32 // hidden


def layer_prefix(index: int) -> str:
    return f"language_model.model.layers.{index}.mlp"


def moe_layers(store: SafeTensorStore) -> List[int]:
    """Indices of the decoder layers that carry a routed expert block."""
    out = []
    for name in store.refs:
        if name.endswith(".mlp.switch_mlp.gate_proj.weight") and name.startswith("language_model.model.layers."):
            out.append(int(name.split(".")[3]))
    return sorted(out)


def _proj(store: SafeTensorStore, prefix: str, device, native: bool = False) -> "ops.Q4Projection":
    """One 4-bit projection; a coarser grouping (64, 128 ...) is expanded to
    the kernels' groups of 32 (Q4Projection.from_group), except groups of 64
    when `native` is set, which stay as stored."""
    inputs = int(store.shape(f"{prefix}.weight")[-1]) * 8
    groups = int(store.shape(f"{prefix}.scales")[-1])
    if groups <= 0 or inputs % groups:
        raise ValueError(f"{prefix}: {inputs} inputs do not split into {groups} groups")
    return ops.Q4Projection.from_group(store.tensor(f"{prefix}.weight", device),
                                       store.tensor(f"{prefix}.scales", device),
                                       store.tensor(f"{prefix}.biases", device), inputs // groups,
                                       native=native)


def load_moe_layer(store: SafeTensorStore, index: int, top_k: int, device=None,
                   pack: bool = True, native_groups: bool = True) -> "ops.MoEWeights":
    """The routed MoE block of decoder layer `index` as MoEWeights (routed
    experts, shared expert and its gate, router), packed into the tiled pool
    unless `pack` is False.  `top_k` is the model's num_experts_per_tok.
    With `native_groups` a G64 layer keeps its scale/bias pairs as stored
    (half the metadata bytes; always packed, the kernels read G64 from the
    tiled records only); otherwise they are expanded to groups of 32."""
    device = torch.device(device) if device is not None else torch.device("cuda")
    mlp = layer_prefix(index)
    sw = f"{mlp}.switch_mlp"
    if f"{sw}.gate_proj.weight" not in store:
        raise KeyError(f"layer {index} has no routed expert block")
    group, bits = infer_switch_quantization(store, sw)
    if bits != 4 or group % 32:
        raise ValueError(f"layer {index}: {bits}-bit codes in groups of {group}; the kernels take 4-bit "
                         "codes in groups of a multiple of 32")
    shared = f"{mlp}.shared_expert.gate_proj.weight" in store
    # native only when every bank bound for the tiled pool (routed, and the
    # shared expert stored beside them) has groups of 64
    nat = native_groups and group == ops.NATIVE_GROUP
    for q in [f"{sw}.{part}" for part in ("gate_proj", "up_proj", "down_proj")] + \
            ([f"{mlp}.shared_expert.{part}" for part in ("gate_proj", "up_proj", "down_proj")]
             if shared else []):
        inputs = int(store.shape(f"{q}.weight")[-1]) * 8
        nat = nat and int(store.shape(f"{q}.scales")[-1]) * group == inputs
    w = ops.MoEWeights(
        _proj(store, f"{sw}.gate_proj", device, nat), _proj(store, f"{sw}.up_proj", device, nat),
        _proj(store, f"{sw}.down_proj", device, nat),
        router_w=store.tensor(f"{mlp}.gate.weight", device),
        shared_gate=_proj(store, f"{mlp}.shared_expert.gate_proj", device, nat) if shared else None,
        shared_up=_proj(store, f"{mlp}.shared_expert.up_proj", device, nat) if shared else None,
        shared_down=_proj(store, f"{mlp}.shared_expert.down_proj", device, nat) if shared else None,
        shared_expert_gate=(_proj(store, f"{mlp}.shared_expert_gate", device)
                            if f"{mlp}.shared_expert_gate.weight" in store else None),
        top_k=top_k, device=device)
    return w.pack() if pack and w.pool is None else w


# --------------------------------------------------------------------------
# Writing (tests and tools that produce a checkpoint-shaped file)
# --------------------------------------------------------------------------

_NP_TO_ST = {np.dtype(np.uint32): "U32", np.dtype(np.int32): "I32", np.dtype(np.float16): "F16",
             np.dtype(np.float32): "F32", np.dtype(np.uint8): "U8"}


def save_safetensors(path: str, tensors: Dict[str, np.ndarray], bf16: Sequence[str] = ()) -> None:
    """Write numpy arrays as a .safetensors file; names in `bf16` are uint16
    bit patterns stored as BF16."""
    header, blobs, off = {}, [], 0
    for name, arr in tensors.items():
        arr = np.ascontiguousarray(arr)
        if name in bf16:
            if arr.dtype != np.uint16:
                raise TypeError(f"{name}: bf16 tensors are passed as uint16 bit patterns")
            dtype = "BF16"
        else:
            dtype = _NP_TO_ST[arr.dtype]
        raw = arr.tobytes()
        header[name] = {"dtype": dtype, "shape": list(arr.shape), "data_offsets": [off, off + len(raw)]}
        blobs.append(raw)
        off += len(raw)
    head = json.dumps(header).encode()
    head += b" " * ((8 - len(head) % 8) % 8)
    with open(path, "wb") as fh:
        fh.write(struct.pack("<Q", len(head)))
        fh.write(head)
        for raw in blobs:
            fh.write(raw)
