"""The tiled expert pool on the GPU: the packing kernel writes the oracle's
record layout byte for byte, and every entry point that streams the pool
returns the same routing as the same weights in the MLX layout and outputs
that differ only by float32 summation (the tiled gate/up GEMV unpacks to f16
q * 2^-24 against power-of-two-scaled activations, the MLX-layout kernel to
bf16 128 + q: the same exact products), and stays within the oracle
tolerance."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import vxmoe_oracle as O
from helpers import assert_same_products, bank_t, bf16_t, np32, weights_from_oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.fail("GPU tests need a CUDA device")
    import vxmoe
    vxmoe._lib.load()


def _bits(t):
    return t.view(torch.int16).cpu().numpy()


@pytest.mark.parametrize("E,out,inn,tr,pair", [
    (3, 40, 96, 16, True), (2, 70, 160, 32, False), (2, 24, 32, 16, False),
    (4, 512, 2048, 16, True), (4, 2048, 512, 32, False)])
def test_pack_kernel_writes_the_oracle_layout(E, out, inn, tr, pair):
    from vxmoe.ops import Q4Projection, tile_bank
    rng = np.random.default_rng(E + out + inn)
    a = O.make_q4_bank(rng, E, out, inn)
    b = O.make_q4_bank(rng, E, out, inn) if pair else None
    rec = tile_bank(Q4Projection(*bank_t(a)), Q4Projection(*bank_t(b)) if pair else None, tr)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(rec.cpu().numpy(), O.tile_records(a, b, tr))


def _pair(p, shared=True, down_rows=32):
    plain = weights_from_oracle(p, shared=shared)
    tiled = weights_from_oracle(p, shared=shared).pack(down_rows)
    return plain, tiled


@pytest.mark.parametrize("cfg", [
    dict(seed=11, experts=32, hidden=256, inter=64, shared_inter=64, top_k=4),
    dict(seed=12, experts=16, hidden=160, inter=96, shared_inter=32, top_k=3),   # ragged chunks
    dict(seed=13, experts=24, hidden=512, inter=160, shared_inter=224, top_k=8),  # Is != I
])
@pytest.mark.parametrize("down_rows", [32, 16])
def test_tiled_block_matches_mlx_layout(cfg, down_rows):
    import vxmoe
    p = O.make_params(**cfg)
    plain, tiled = _pair(p, down_rows=down_rows)
    for T in (1, 2, 7, 40):
        x = bf16_t(O.make_x(30 + T, T, p.hidden))
        y0, i0, w0 = vxmoe.moe_block(x, plain, return_routing=True)
        y1, i1, w1 = vxmoe.moe_block(x, tiled, return_routing=True)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(i0.cpu().numpy(), i1.cpu().numpy())
        np.testing.assert_array_equal(_bits(w0), _bits(w1))
        assert_same_products(y1, y0, f"T={T}")


def test_tiled_block_rows_of_wide_range():
    """All activation records of a position share one power-of-two scale,
    chosen from the row's largest |x|: chunks 2^32 smaller than the row's
    largest meet f16 subnormals, whose terms sit far below the float32 sums'
    rounding, so the tiled block still matches the MLX-layout block and the
    oracle.  Zero chunks and an all-zero row take scale 1.  T > 4 runs the
    records pass (smaller batches take the single-launch decode kernel)."""
    import vxmoe
    p = O.make_params(seed=14, experts=16, hidden=512, inter=128, shared_inter=64, top_k=4)
    plain, tiled = _pair(p)
    for T in (5, 40):
        x = O.make_x(60 + T, T, p.hidden).copy()
        x[:, :128] *= 2.0 ** 8
        x[:, 128:256] *= 2.0 ** -24
        x[1::3, 256:384] = 0.0
        x[2] = 0.0
        xt = bf16_t(x)
        y0, i0, _ = vxmoe.moe_block(xt, plain, return_routing=True)
        y1, i1, _ = vxmoe.moe_block(xt, tiled, return_routing=True)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(i0.cpu().numpy(), i1.cpu().numpy())
        assert_same_products(y1, y0, f"wide-range rows, T={T}")
        assert np.all(np.isfinite(np32(y1)))
        logits = np32(vxmoe.router(xt, tiled).logits)
        out = O.moe_block(np32(xt), p, logits=logits)
        assert O.normwise_error(np32(y1), out.y) < 1e-2, f"T={T}"


def test_tiled_block_production_against_oracle():
    import vxmoe
    p = O.make_params(seed=0)
    w = weights_from_oracle(p).pack()
    for T in (1, 8):
        x = O.make_x(1, T, 2048)
        y, inds, _ = vxmoe.moe_block(bf16_t(x), w, return_routing=True)
        logits = np32(vxmoe.router(bf16_t(x), w).logits)
        out = O.moe_block(x, p, logits=logits)
        np.testing.assert_array_equal(inds.cpu().numpy(), out.router.inds)
        assert O.normwise_error(np32(y), out.y) < 1e-2
        ref = O.moe_block_reference_f64(x, p, out.router.inds, out.router.logits)
        assert O.normwise_error(np32(y), ref) <= 1.5 * O.normwise_error(out.y, ref) + 2e-3


def test_tiled_executor_paths_match_mlx_layout():
    import vxmoe
    p = O.make_params(seed=21, experts=32, hidden=256, inter=64, shared_inter=64, top_k=4)
    plain, tiled = _pair(p, shared=False)
    T = 9
    x = bf16_t(O.make_x(5, T, p.hidden))
    rng = np.random.default_rng(3)
    routes = torch.from_numpy(rng.integers(0, p.num_experts, (T, p.top_k)).astype(np.int32)).cuda()
    scores = bf16_t(O.bf16_round(rng.random((T, p.top_k)).astype(np.float32)))
    for kw in (dict(), dict(scores=scores)):
        a = vxmoe.moe_experts(x, routes, plain, **kw)
        b = vxmoe.moe_experts(x, routes, tiled, **kw)
        torch.cuda.synchronize()
        assert_same_products(b, a, f"moe_experts {sorted(kw)}")
    half = torch.where(routes < 16, routes, torch.full_like(routes, -1))
    a = vxmoe.moe_experts_partial(x, half, scores, plain)
    b = vxmoe.moe_experts_partial(x, half, scores, tiled)
    torch.cuda.synchronize()
    assert_same_products(b, a, "moe_experts_partial")


def test_pool_shape_mismatch_is_rejected():
    import vxmoe
    p = O.make_params(seed=11, experts=32, hidden=256, inter=64, shared_inter=64, top_k=4)
    w = weights_from_oracle(p).pack()
    w.pool.vx().down.tile_rows = 8
    with pytest.raises(ValueError):
        vxmoe.moe_block(bf16_t(O.make_x(1, 2, p.hidden)), w)
