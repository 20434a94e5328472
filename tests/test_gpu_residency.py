"""Partial residency on the device (vxmoe.SlotPool): a layer whose routed
records live in pinned host memory and reach a shared device pool of expert
slots on demand gives the bits of the same layer fully resident - the
kernels read the same records through the slot table (vx_moe_pool.slot_of)
- through the single-launch decode kernel, the multi-kernel GEMV pipeline
and the tcgen05 GEMM; two layers sharing a pool smaller than one layer's
bank evict each other's experts and still reproduce their own outputs."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import vxmoe_oracle as O
from helpers import bf16_t, weights_from_oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.fail("GPU tests need a CUDA device")
    import vxmoe
    vxmoe._lib.load()


def _bits(t):
    return t.view(torch.int16).cpu().numpy()


def _same(a, b, what):
    np.testing.assert_array_equal(_bits(a), _bits(b), err_msg=what)


def test_slot_pool_layer_equals_resident_layer():
    import vxmoe
    from vxmoe import _lib
    p = O.make_params(seed=0)
    full = weights_from_oracle(p).pack()
    part = weights_from_oracle(p)
    pool = vxmoe.SlotPool(48, p.hidden, p.gate.w.shape[1])
    pool.attach(part)
    assert not part.gate.weight.is_cuda          # the routed banks left the device
    for T in (1, 3, 4):
        x = bf16_t(O.make_x(70 + T, T, p.hidden))
        _same(vxmoe.moe_block(x, part), vxmoe.moe_block(x, full), f"decode kernel T={T}")
        for w in (part, full):
            w.expert_path = _lib.PATH_GEMV
        try:
            _same(vxmoe.moe_block(x, part), vxmoe.moe_block(x, full), f"GEMV pipeline T={T}")
        finally:
            for w in (part, full):
                w.expert_path = _lib.PATH_AUTO
    assert pool.assigner.misses > 0 and pool.assigner.hits > 0


def test_two_layers_share_a_small_pool():
    import vxmoe
    pa, pb = O.make_params(seed=0), O.make_params(seed=1)
    fa, fb = weights_from_oracle(pa).pack(), weights_from_oracle(pb).pack()
    la, lb = weights_from_oracle(pa), weights_from_oracle(pb)
    pool = vxmoe.SlotPool(24, pa.hidden, pa.gate.w.shape[1])   # less than one layer's 512 experts
    pool.attach(la)
    pool.attach(lb)
    g = torch.Generator(device="cuda")
    g.manual_seed(9)
    for step in range(6):
        x = torch.randn((2, pa.hidden), device="cuda", generator=g).to(torch.bfloat16)
        _same(vxmoe.moe_block(x, la), vxmoe.moe_block(x, fa), f"layer A step {step}")
        _same(vxmoe.moe_block(x, lb), vxmoe.moe_block(x, fb), f"layer B step {step}")
    assert pool.assigner.misses > pool.slots     # experts were evicted and refilled


def test_slot_pool_prefill_gemm():
    import vxmoe
    from vxmoe import _lib
    p = O.make_params(seed=3, experts=64, hidden=256, inter=128, shared_inter=128, top_k=4)
    full = weights_from_oracle(p).pack()
    part = weights_from_oracle(p)
    pool = vxmoe.SlotPool(64, p.hidden, p.gate.w.shape[1])
    pool.attach(part)
    for w in (part, full):
        w.expert_path = _lib.PATH_GEMM
    x = bf16_t(O.make_x(3, 96, p.hidden))
    _same(vxmoe.moe_block(x, part), vxmoe.moe_block(x, full), "tcgen05 GEMM")
    # experts land in slots in first-use order, not at their own index
    slots = [pool.assigner.slot(part.slot_layer, e) for e in range(p.num_experts)]
    assert any(s is not None and s != e for e, s in enumerate(slots))
