"""A layer loaded from a checkpoint-shaped safetensors file runs the block
with the same bits as the same weights built in memory, and the block works at
the real checkpoint's width (d=2560, I=Is=640, models/flashnext/preflight.py:
53-56) within the block tolerance of the oracle."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import vxmoe_oracle as O
from helpers import bf16_t, np32, weights_from_oracle
from test_loader_cpu import checkpoint_tensors

pytestmark = pytest.mark.gpu


def test_loaded_layer_equals_in_memory_weights(tmp_path):
    import vxmoe
    from vxmoe import loader as L
    p = O.make_params(seed=61, experts=32, hidden=512, inter=256, shared_inter=128, top_k=4)
    tensors, bf16 = checkpoint_tensors(p, 5)
    path = str(tmp_path / "model.safetensors")
    L.save_safetensors(path, tensors, bf16=bf16)
    store = L.SafeTensorStore([path])
    w = L.load_moe_layer(store, 5, top_k=p.top_k, device="cuda")
    ref_w = weights_from_oracle(p).pack()
    for T in (1, 7, 64):
        x = bf16_t(O.make_x(62 + T, T, p.hidden))
        y = vxmoe.moe_block(x, w)
        ref = vxmoe.moe_block(x, ref_w)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(y.view(torch.int16).cpu().numpy(), ref.view(torch.int16).cpu().numpy())


def test_g64_layer_runs_within_tolerance(tmp_path):
    """A G64 checkpoint layer (every projection in groups of 64) loads with
    native G64 records (the shared-expert gate expanded to groups of 32):
    routing bit-exact against the oracle on the device's logits, outputs
    within the block tolerance of the G64 oracle, and the bits of the same
    layer loaded with every group expanded to 32."""
    import vxmoe
    from vxmoe import loader as L
    p = O.make_params(seed=63, experts=32, hidden=512, inter=256, shared_inter=128, top_k=4, group_size=64)
    tensors, bf16 = checkpoint_tensors(p, 2)
    path = str(tmp_path / "g64.safetensors")
    L.save_safetensors(path, tensors, bf16=bf16)
    store = L.SafeTensorStore([path])
    assert L.infer_switch_quantization(store, L.layer_prefix(2) + ".switch_mlp") == (64, 4)
    w = L.load_moe_layer(store, 2, top_k=p.top_k, device="cuda")
    assert w.group_size == 64 and w.pool.group_size == 64
    assert w.shared_expert_gate.group_size == 32
    w32 = L.load_moe_layer(store, 2, top_k=p.top_k, device="cuda", native_groups=False)
    assert w32.group_size == 32
    for T in (3, 200):   # decode GEMV and prefill GEMM
        x = O.make_x(66 + T, T, p.hidden)
        y, inds, _ = vxmoe.moe_block(bf16_t(x), w, return_routing=True)
        logits = np32(vxmoe.router(bf16_t(x), w).logits)
        out = O.moe_block(x, p, logits=logits, path="prefill" if T > 3 else "decode")
        np.testing.assert_array_equal(inds.cpu().numpy(), out.router.inds)
        assert O.normwise_error(np32(y), out.y) < 1e-2
        if T > 3:   # the GEMM path; decode-sized G32 batches take the decode kernel
            y32 = vxmoe.moe_block(bf16_t(x), w32)
            np.testing.assert_array_equal(y.view(torch.int16).cpu().numpy(),
                                          y32.view(torch.int16).cpu().numpy())


def test_8bit_layer_is_refused(tmp_path):
    from vxmoe import loader as L
    p = O.make_params(seed=63, experts=8, hidden=256, inter=128, shared_inter=64, top_k=2)
    tensors, bf16 = checkpoint_tensors(p, 0)
    name = L.layer_prefix(0) + ".switch_mlp.gate_proj.weight"
    tensors[name] = np.zeros((8, 128, 256 // 4), np.uint32)   # four codes per word: 8-bit
    path = str(tmp_path / "q8.safetensors")
    L.save_safetensors(path, tensors, bf16=bf16)
    with pytest.raises(ValueError):
        L.load_moe_layer(L.SafeTensorStore([path]), 0, top_k=2, device="cuda")


@pytest.mark.parametrize("T", [1, 16, 300])
def test_block_at_checkpoint_width(T):
    """d=2560, I=640 (40 row tiles of the pool, 20 and 5 chunks of 128
    inputs): decode GEMV and prefill GEMM paths against the oracle."""
    import vxmoe
    p = O.make_params(seed=64, experts=64, hidden=2560, inter=640, shared_inter=640, top_k=10)
    w = weights_from_oracle(p).pack()
    x = O.make_x(65, T, p.hidden)
    y, inds, _ = vxmoe.moe_block(bf16_t(x), w, return_routing=True)
    logits = np32(vxmoe.router(bf16_t(x), w).logits)
    out = O.moe_block(x, p, logits=logits)
    np.testing.assert_array_equal(inds.cpu().numpy(), out.router.inds)
    assert O.normwise_error(np32(y), out.y) < 1e-2
