"""The checkpoint reader (vxmoe.loader): a synthetic safetensors file with the
reference's tensor names (models/flashnext/preflight.py:68-75) round-trips,
the per-layer quantization is inferred from the shapes as
models/flashnext/loader.py:379-401 does, and malformed files are rejected."""
from __future__ import annotations

import json
import struct

import numpy as np
import pytest

import vxmoe_oracle as O
from vxmoe import loader as L


def checkpoint_tensors(p: "O.MoEParams", layer: int, group_override=None):
    """The MoE tensors of one decoder layer, named as the reference checkpoint
    names them; bf16 values as uint16 bit patterns."""
    mlp = L.layer_prefix(layer)
    out, bf16 = {}, []

    def bank(name, b: "O.Q4Bank"):
        out[f"{name}.weight"] = b.w.astype(np.uint32)
        out[f"{name}.scales"] = O.bf16_bits(b.scales)
        out[f"{name}.biases"] = O.bf16_bits(b.biases)
        bf16.extend([f"{name}.scales", f"{name}.biases"])

    bank(f"{mlp}.switch_mlp.gate_proj", p.gate)
    bank(f"{mlp}.switch_mlp.up_proj", p.up)
    bank(f"{mlp}.switch_mlp.down_proj", p.down)
    bank(f"{mlp}.shared_expert.gate_proj", p.shared_gate)
    bank(f"{mlp}.shared_expert.up_proj", p.shared_up)
    bank(f"{mlp}.shared_expert.down_proj", p.shared_down)
    bank(f"{mlp}.shared_expert_gate", p.shared_expert_gate)
    out[f"{mlp}.gate.weight"] = O.bf16_bits(p.router_w)
    bf16.append(f"{mlp}.gate.weight")
    if group_override:   # scales/biases of a coarser grouping on the gate projection
        g = group_override
        name = f"{mlp}.switch_mlp.gate_proj"
        out[f"{name}.scales"] = out[f"{name}.scales"][..., ::g // 32].copy()
        out[f"{name}.biases"] = out[f"{name}.biases"][..., ::g // 32].copy()
    return out, bf16


def small_params(seed=7):
    return O.make_params(seed=seed, experts=8, hidden=256, inter=128, shared_inter=64, top_k=2)


def test_round_trip_and_quantization(tmp_path):
    p = small_params()
    tensors, bf16 = checkpoint_tensors(p, 3)
    extra = {"language_model.model.layers.0.input_layernorm.weight": np.ones(256, np.uint16)}
    path = str(tmp_path / "model-00001.safetensors")
    L.save_safetensors(path, {**extra, **tensors}, bf16=bf16 + list(extra))
    store = L.SafeTensorStore.from_dir(str(tmp_path))
    assert L.moe_layers(store) == [3]
    for name, arr in tensors.items():
        assert store.shape(name) == arr.shape
        np.testing.assert_array_equal(store.numpy(name), arr)
    assert L.infer_switch_quantization(store, L.layer_prefix(3) + ".switch_mlp") == (32, 4)


def test_group64_layout_is_inferred(tmp_path):
    p = small_params()
    tensors, bf16 = checkpoint_tensors(p, 0, group_override=64)
    path = str(tmp_path / "g64.safetensors")
    L.save_safetensors(path, tensors, bf16=bf16)
    store = L.SafeTensorStore([path])
    assert L.infer_switch_quantization(store, L.layer_prefix(0) + ".switch_mlp") == (64, 4)


def test_incompatible_shapes_rejected(tmp_path):
    p = small_params()
    tensors, bf16 = checkpoint_tensors(p, 0)
    name = L.layer_prefix(0) + ".switch_mlp.gate_proj.scales"
    tensors[name] = tensors[name][..., :5].copy()        # 256 inputs in 5 groups
    path = str(tmp_path / "bad.safetensors")
    L.save_safetensors(path, tensors, bf16=bf16)
    store = L.SafeTensorStore([path])
    with pytest.raises(ValueError):
        L.infer_switch_quantization(store, L.layer_prefix(0) + ".switch_mlp")


def test_malformed_files_rejected(tmp_path):
    bad = tmp_path / "short.safetensors"
    bad.write_bytes(b"\x01\x02")
    with pytest.raises(ValueError):
        L.SafeTensorStore([str(bad)])
    head = json.dumps({"t": {"dtype": "F32", "shape": [4], "data_offsets": [0, 12]}}).encode()
    wrong = tmp_path / "offsets.safetensors"
    wrong.write_bytes(struct.pack("<Q", len(head)) + head + b"\0" * 16)
    with pytest.raises(ValueError):
        L.SafeTensorStore([str(wrong)])
    huge = tmp_path / "huge.safetensors"
    huge.write_bytes(struct.pack("<Q", L.HEADER_LIMIT + 1) + b"{}")
    with pytest.raises(ValueError):
        L.SafeTensorStore([str(huge)])
