"""Adaptive top-k on the device (threshold < 1.0, adaptive_topk.py:44-51,
:107-118, :224-233): a token keeps its leading slots until they hold the
threshold's share of its top-k probability mass (at least min_keep); its
other slots name its first expert with weight 0, and the weights
renormalise over the kept mass.  Checked: ids bit-exact and weights within
2 bf16 ulp of the oracle run on the device's own logits, through the fused
router, the tiled prefill router (equal to the fused one bit for bit), the
single-launch decode kernel (equal to the multi-kernel pipeline) and the
block output against the oracle bar; fewer distinct experts are read."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import vxmoe_oracle as O
from helpers import assert_block_bar, assert_same_products, bf16_t, np32, ulp_diff_bf16, weights_from_oracle

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


class _Keep:
    def __init__(self, w, threshold, min_keep=1):
        self.w, self.t, self.m = w, threshold, min_keep

    def __enter__(self):
        self.w.threshold, self.w.min_keep = self.t, self.m

    def __exit__(self, *a):
        self.w.threshold, self.w.min_keep = 1.0, 1


@pytest.mark.parametrize("threshold,min_keep", [(0.9, 1), (0.7, 3), (0.5, 1)])
def test_router_adaptive_matches_oracle(prod, threshold, min_keep):
    import vxmoe
    p, w = prod
    x = bf16_t(O.make_x(40, 64, p.hidden))
    with _Keep(w, threshold, min_keep):
        r = vxmoe.router(x, w)
    torch.cuda.synchronize()
    own = O.router(None, None, p.top_k, logits=np32(r.logits), threshold=threshold, min_keep=min_keep)
    np.testing.assert_array_equal(r.inds.cpu().numpy(), own.inds)
    assert ulp_diff_bf16(np32(r.weights), own.weights).max() <= 2
    keeps = O.keeps_of(own.inds)
    assert keeps.min() >= min_keep and keeps.mean() < p.top_k
    assert np.all(np32(r.weights)[np.arange(p.top_k)[None, :] >= keeps[:, None]] == 0)


def test_router_adaptive_tiled_equals_fused(prod):
    import vxmoe
    p, w = prod
    x = bf16_t(O.make_x(41, 600, p.hidden))
    with _Keep(w, 0.8):
        whole = vxmoe.router(x, w)
        parts = [vxmoe.router(x[a:a + 200], w) for a in (0, 200, 400)]
    torch.cuda.synchronize()
    for name in ("inds", "weights"):
        got = getattr(whole, name)
        exp = torch.cat([getattr(r, name) for r in parts])
        assert torch.equal(got.view(torch.int16) if got.dtype == torch.bfloat16 else got,
                           exp.view(torch.int16) if exp.dtype == torch.bfloat16 else exp), name


@pytest.mark.parametrize("T", [1, 4, 16])
def test_block_adaptive_against_oracle(prod, T):
    import vxmoe
    from vxmoe import _lib
    p, w = prod
    x_np = O.make_x(950 + T, T, p.hidden)
    x = bf16_t(x_np)
    with _Keep(w, 0.85):
        y, inds, wts = vxmoe.moe_block(x, w, return_routing=True)
        if T <= 4:   # the single-launch decode kernel against the multi-kernel pipeline
            w.expert_path = _lib.PATH_GEMV
            try:
                y2, inds2, wts2 = vxmoe.moe_block(x, w, return_routing=True)
            finally:
                w.expert_path = _lib.PATH_AUTO
            torch.cuda.synchronize()
            np.testing.assert_array_equal(inds.cpu().numpy(), inds2.cpu().numpy())
            np.testing.assert_array_equal(O.bf16_bits(np32(wts)), O.bf16_bits(np32(wts2)))
            assert_same_products(y, y2, f"adaptive T={T}")
    logits = np32(vxmoe.router(x, w).logits)   # the logits do not depend on the threshold
    out = O.moe_block(x_np, p, logits=logits, threshold=0.85)
    np.testing.assert_array_equal(inds.cpu().numpy(), out.router.inds)
    keeps = O.keeps_of(out.router.inds)
    ref64 = O.moe_block_reference_f64(x_np, p, out.router.inds, out.router.logits, keeps=keeps)
    scale = O.summand_scale(out.yd, out.router.weights, out.shared_y)
    assert_block_bar(np32(y), out.y, ref64, scale, f"adaptive 0.85 T={T}")
    exact = O.router(None, None, p.top_k, logits=logits)
    assert len(np.unique(out.router.inds)) <= len(np.unique(exact.inds))
