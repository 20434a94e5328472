"""The single-launch decode kernel (vx_decode.cu): a block call of at most four
tokens over the tiled pool runs router, top-k, expert sort, gate/up, down and
combine in one cooperative launch.

Checked here against the multi-kernel pipeline (the same weights with the
expert path forced to the grouped GEMV kernels) and against the oracle:
routing (ids and renormalised weights) equal to the standalone router's bit
for bit, so the logits are the same; block outputs within the block bar of
the oracle and close to the multi-kernel pipeline (the same arithmetic, the
chunk partial sums of a task added in another order);
batches with and without the shared expert, with the skew benchmark's router
bias, both down tilings of the pool, and replay inside a CUDA graph.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import vxmoe_oracle as O
from helpers import assert_block_bar, assert_same_products, bf16_t, np32, weights_from_oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.fail("GPU tests need a CUDA device")
    import vxmoe
    vxmoe._lib.load()


@pytest.fixture(scope="module")
def prod():
    p = O.make_params(seed=0)
    return p, weights_from_oracle(p).pack()


def _multi_kernel(w, x):
    """The same block through the multi-kernel pipeline (router, expert sort,
    grouped GEMVs, combine)."""
    import vxmoe
    from vxmoe import _lib
    old = w.expert_path
    w.expert_path = _lib.PATH_GEMV
    try:
        return vxmoe.moe_block(x, w, return_routing=True)
    finally:
        w.expert_path = old


def _close_to_pipeline(y_dec, y_ref, what):
    """The decode kernel unpacks weights to bf16 128 + q and adds a task's
    per-warp chunk sums at the end; the multi-kernel gate/up GEMV unpacks to
    f16 q * 2^-24 against power-of-two-scaled activations.  Both form the
    same exact products."""
    assert_same_products(y_dec, y_ref, what)


@pytest.mark.parametrize("T", [1, 2, 3, 4])
def test_decode_matches_pipeline_and_oracle(prod, T):
    import vxmoe
    p, w = prod
    x_np = O.make_x(900 + T, T, p.hidden)
    x = bf16_t(x_np)
    y, inds, wts = vxmoe.moe_block(x, w, return_routing=True)
    y_ref, inds_ref, wts_ref = _multi_kernel(w, x)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(inds.cpu().numpy(), inds_ref.cpu().numpy())
    np.testing.assert_array_equal(O.bf16_bits(np32(wts)), O.bf16_bits(np32(wts_ref)))
    _close_to_pipeline(y, y_ref, f"T={T}")
    logits = np32(vxmoe.router(x, w).logits)
    out = O.moe_block(x_np, p, logits=logits)
    np.testing.assert_array_equal(inds.cpu().numpy(), out.router.inds)
    ref64 = O.moe_block_reference_f64(x_np, p, out.router.inds, out.router.logits)
    scale = O.summand_scale(out.yd, out.router.weights, out.shared_y)
    assert_block_bar(np32(y), out.y, ref64, scale, f"decode T={T}")


def test_decode_routing_equals_router_over_many_tokens(prod):
    """256 tokens in batches of four (and 96 with the skew bias): the decode
    kernel's ids and weights equal the standalone router's bit for bit."""
    import vxmoe
    p, w = prod
    g = torch.Generator(device="cuda")
    g.manual_seed(5)
    hot = np.random.default_rng(0).choice(p.num_experts, 32, replace=False)
    bias = np.zeros(p.num_experts, np.float32)
    bias[hot] = 2.0
    for use_bias, n in ((False, 64), (True, 24)):
        w.router_bias = bf16_t(bias) if use_bias else None
        try:
            for _ in range(n):
                x = torch.randn((4, p.hidden), device="cuda", generator=g).to(torch.bfloat16)
                _, inds, wts = vxmoe.moe_block(x, w, return_routing=True)
                r = vxmoe.router(x, w)
                assert torch.equal(inds, r.inds)
                assert torch.equal(wts.view(torch.int16), r.weights.view(torch.int16))
        finally:
            w.router_bias = None


@pytest.mark.parametrize("shared,down_rows", [(False, 32), (True, 16)])
def test_decode_without_shared_and_with_16_row_down_tiles(shared, down_rows):
    import vxmoe
    p = O.make_params(seed=21, experts=128, hidden=1024, inter=256, shared_inter=256, top_k=8)
    w = weights_from_oracle(p, shared=shared).pack(down_rows)
    for T in (1, 3):
        x_np = O.make_x(40 + T, T, p.hidden)
        x = bf16_t(x_np)
        y, inds, wts = vxmoe.moe_block(x, w, return_routing=True)
        y_ref, inds_ref, _ = _multi_kernel(w, x)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(inds.cpu().numpy(), inds_ref.cpu().numpy())
        _close_to_pipeline(y, y_ref, f"shared={shared} rows={down_rows} T={T}")
        logits = np32(vxmoe.router(x, w).logits)
        r = O.router(x_np, p.router_w, p.top_k, logits=logits)
        yd, _ = O.routed_outputs(x_np, r.inds, p)
        if shared:
            sh, sg = O.shared_parts(x_np, p)
            shared_y = O.bf16_round(sg * sh)
        else:
            shared_y = None
        ref = O.fused_combine(yd, r.weights, shared_y)
        assert O.normwise_error(np32(y), ref) < 1e-2


def test_decode_in_a_cuda_graph(prod):
    """The cooperative launch captures into a graph: replays give the eager
    call's bits, for fresh inputs each time."""
    import vxmoe
    p, w = prod
    blk = vxmoe.GraphedBlock(w, 1)
    g = torch.Generator(device="cuda")
    g.manual_seed(11)
    for _ in range(4):
        x = torch.randn((1, p.hidden), device="cuda", generator=g).to(torch.bfloat16)
        y_graph = blk(x).clone()
        y_eager = vxmoe.moe_block(x, w)
        torch.cuda.synchronize()
        assert torch.equal(y_graph.view(torch.int16), y_eager.view(torch.int16))
