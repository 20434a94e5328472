"""The block captured into a CUDA graph replays the same kernels: its output
equals moe_block's bit for bit, call after call, for the decode (tiled GEMV)
and prefill (tcgen05 GEMM) pipelines, and the fused router gives the same
routing as the stand-alone top-k kernel."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import vxmoe_oracle as O
from helpers import bf16_t, np32, weights_from_oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.fail("GPU tests need a CUDA device")


@pytest.mark.parametrize("T,packed", [(8, True), (8, False), (40, True)])
def test_graph_replay_equals_block(T, packed):
    import vxmoe
    p = O.make_params(seed=51, experts=32, hidden=256, inter=128, shared_inter=64, top_k=4)
    w = weights_from_oracle(p)
    if packed:
        w.pack()
    gb = vxmoe.GraphedBlock(w, T)
    for seed in (52, 53):
        x = bf16_t(O.make_x(seed, T, p.hidden))
        ref = vxmoe.moe_block(x, w)
        y = gb(x).clone()
        torch.cuda.synchronize()
        np.testing.assert_array_equal(y.view(torch.int16).cpu().numpy(), ref.view(torch.int16).cpu().numpy())


def test_fused_router_matches_topk_kernel():
    import vxmoe
    p = O.make_params(seed=54, experts=512, hidden=2048, inter=64, shared_inter=64, top_k=10)
    w = weights_from_oracle(p)
    x = bf16_t(O.make_x(55, 37, p.hidden))
    r = vxmoe.router(x, w)
    again = vxmoe.softmax_topk(r.logits, p.top_k)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(r.inds.cpu().numpy(), again.inds.cpu().numpy())
    np.testing.assert_array_equal(r.weights.view(torch.int16).cpu().numpy(),
                                  again.weights.view(torch.int16).cpu().numpy())
    ref = O.router(np32(x), p.router_w, p.top_k, logits=np32(r.logits))
    np.testing.assert_array_equal(r.inds.cpu().numpy(), ref.inds)
