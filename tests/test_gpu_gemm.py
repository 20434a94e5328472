"""The prefill expert path: the grouped tcgen05 GEMM (batches with on average
at least four routed positions per expert) against the oracle's restatement
of MLX's batched quantized matmul (bf16-dequantised tiles, high-precision
sums, bf16 out), at ragged shapes and item sizes, and the whole block
against the float64 reference."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import vxmoe_oracle as O
from helpers import assert_bf16_close, bank_t, bf16_t, np32, weights_from_oracle

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.fail("GPU tests need a CUDA device")
    import vxmoe
    vxmoe._lib.load()


def _per_slot_ref(p, x, routes):
    T, k = routes.shape
    out = np.zeros((T, k, p.hidden), np.float32)
    for e in np.unique(routes):
        tt, ss = np.nonzero(routes == e)
        _, _, _, y = O.expert_mlp_qmm(x[tt], p.gate.expert(e), p.up.expert(e), p.down.expert(e))
        out[tt, ss] = y
    return out


@pytest.mark.parametrize("cfg,T,skew", [
    (dict(seed=31, experts=16, hidden=256, inter=128, shared_inter=32, top_k=4), 16, None),   # 4 per expert
    (dict(seed=32, experts=8, hidden=160, inter=96, shared_inter=32, top_k=2), 40, None),     # ragged K, N
    (dict(seed=33, experts=8, hidden=512, inter=256, shared_inter=32, top_k=3), 150, 0),      # a 150-token expert
    (dict(seed=34, experts=32, hidden=384, inter=224, shared_inter=32, top_k=8), 17, None),   # cnt 17, 33 ...
    # >= 128 positions per expert: the pool kernel's 128-wide items
    (dict(seed=35, experts=8, hidden=256, inter=128, shared_inter=32, top_k=2), 600, None),
    (dict(seed=36, experts=8, hidden=512, inter=256, shared_inter=32, top_k=3), 400, 0),      # 400-token expert
])
@pytest.mark.parametrize("packed", [False, True])
def test_gemm_per_slot_outputs_match_qmm_oracle(cfg, T, skew, packed):
    import vxmoe
    p = O.make_params(**cfg)
    rng = np.random.default_rng(cfg["seed"])
    routes = np.stack([rng.permutation(p.num_experts)[:p.top_k] for _ in range(T)]).astype(np.int32)
    if skew is not None:
        routes[:, 0] = skew                        # every token also visits expert `skew`
    x = O.make_x(cfg["seed"] + 1, T, p.hidden)
    w = weights_from_oracle(p, shared=False)
    if packed:                                     # the persistent kernel over the tiled pool
        w.pack(down_rows=32 if cfg["seed"] % 2 else 16)
    assert T * p.top_k >= 4 * p.num_experts        # the GEMM path
    out = vxmoe.moe_experts(bf16_t(x), torch.from_numpy(routes).cuda(), w)
    torch.cuda.synchronize()
    ref = _per_slot_ref(p, x, routes)
    # h is rounded to bf16 between the two GEMMs; where the float32 tensor-core
    # sum and the float64 oracle sum round h differently (1 ulp), the down
    # output moves by ~1e-3 of its rms - many ulps for outputs near zero (the
    # more tokens, the more such outliers: 5 ulps at 8 % of the rms at T=600,
    # 32 ulps at 3 % of the rms - 0.5 % of the rms absolute - at T=400, where
    # the array and the pool kernels agree with each other bit for bit).
    assert_bf16_close(np32(out), ref, max_ulp=2, min_exact=0.9, floor=2.0 ** -7,
                      what=f"gemm per-slot T={T}")
    assert O.normwise_error(np32(out), ref) < 4e-3


@pytest.mark.parametrize("packed", [False, True])
def test_gemm_block_matches_float64_reference(packed):
    import vxmoe
    p = O.make_params(seed=41, experts=64, hidden=512, inter=256, shared_inter=256, top_k=8)
    T = 64                                         # 8 routed positions per expert on average
    x = O.make_x(42, T, p.hidden)
    w = weights_from_oracle(p)
    if packed:
        w.pack()
    y, inds, _ = vxmoe.moe_block(bf16_t(x), w, return_routing=True)
    logits = np32(vxmoe.router(bf16_t(x), w).logits)
    out = O.moe_block(x, p, logits=logits)
    np.testing.assert_array_equal(inds.cpu().numpy(), out.router.inds)
    got = np32(y)
    assert O.normwise_error(got, out.y) < 1e-2
    ref = O.moe_block_reference_f64(x, p, out.router.inds, out.router.logits)
    assert O.normwise_error(got, ref) <= 1.5 * O.normwise_error(out.y, ref) + 2e-3


@pytest.mark.parametrize("T", [32, 600])   # 600 tokens: 150 positions per expert, 128-wide items
def test_gemm_block_pool_kernel_matches_array_kernel(T):
    """The persistent kernel over the tiled pool and the kernel reading the MLX
    arrays dequantise identically; the pool kernel sums the down projection
    in two interleaved accumulators (even and odd 64-input blocks), so the
    float32 sums may round differently: within one bf16 ulp, rarely two (seen
    at T=600)."""
    import vxmoe
    from helpers import ulp_diff_bf16
    p = O.make_params(seed=43, experts=16, hidden=256, inter=128, shared_inter=64, top_k=4)
    x = bf16_t(O.make_x(44, T, p.hidden))
    a = vxmoe.moe_block(x, weights_from_oracle(p))
    b = vxmoe.moe_block(x, weights_from_oracle(p).pack())
    torch.cuda.synchronize()
    d = ulp_diff_bf16(np32(a), np32(b))
    assert d.max() <= 2 and float(np.mean(d <= 1)) > 0.9999 and float(np.mean(d == 0)) > 0.97


@pytest.mark.slow
def test_gemm_production_prefill_shape():
    """C4-like: production layer, 256 tokens (5 positions per expert)."""
    import vxmoe
    p = O.make_params(seed=0)
    T = 256
    x = O.make_x(45, T, 2048)
    w = weights_from_oracle(p).pack()              # the benchmark's layout
    y, inds, wts = vxmoe.moe_block(bf16_t(x), w, return_routing=True)
    logits = np32(vxmoe.router(bf16_t(x), w).logits)
    r = O.router(x, p.router_w, p.top_k, logits=logits)
    np.testing.assert_array_equal(inds.cpu().numpy(), r.inds)
    shared, sg = O.shared_parts(x, p)
    yd = _per_slot_ref(p, x, r.inds)
    ref = O.fused_combine(yd, r.weights, O.bf16_round(sg * shared))
    assert O.normwise_error(np32(y), ref) < 1e-2
