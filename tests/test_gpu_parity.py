"""Parity of the CUDA path with the CPU oracle (needs a B200).

Bar: bit-exact for nibble unpack, dequantised weights, the bf16 SwiGLU
contract, top-k expert ids and the permutation; bf16 outputs of float
accumulations within one bf16 ulp of the oracle (float32 vs float64 sums);
block outputs within 1e-2 of the oracle (max relative error with each
output's denominator floored at the magnitude of the terms it sums; and
normwise), no further from the unrounded float64 reference than the oracle's
own bf16 semantics are, and allclose(atol=rtol=1e-2) against both
(helpers.assert_block_bar).
"""
from __future__ import annotations

import os

import numpy as np
import pytest
import torch

import vxmoe_oracle as O
from helpers import (assert_block_bar, assert_bf16_close, bank_t, bf16_t, np32, u32_t,
                     ulp_diff_bf16, weights_from_oracle)

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.fail("GPU tests need a CUDA device")
    import vxmoe
    vxmoe._lib.load()


@pytest.fixture(scope="module")
def small_params():
    return O.make_params(seed=11, experts=32, hidden=256, inter=64, shared_inter=64, top_k=4)


@pytest.fixture(scope="module")
def prod_params():
    return O.make_params(seed=0)


# ---------------------------------------------------------------- Q4 pieces

def test_dequant_bit_exact_vs_reference_golden(golden_dir):
    import vxmoe
    g = np.load(os.path.join(golden_dir, "dequant.npz"))
    for e in range(g["w"].shape[0]):
        out = vxmoe.dequantize(u32_t(g["w"]), bf16_t(g["scales"]), bf16_t(g["biases"]), expert=e)
        np.testing.assert_array_equal(np32(out).view(np.uint32), g["dequant"][e].view(np.uint32))


def test_dequant_bit_exact_production_expert(prod_params):
    import vxmoe
    b = prod_params.down
    for e in (0, 511):
        out = vxmoe.dequantize(u32_t(b.w), bf16_t(b.scales), bf16_t(b.biases), expert=e)
        ref = O.dequantize(b.w[e], b.scales[e], b.biases[e])
        np.testing.assert_array_equal(np32(out).view(np.uint32), ref.view(np.uint32))


def test_swiglu_bf16_contract_exhaustive():
    import vxmoe
    gate = O.bf16_from_bits(np.arange(65536, dtype=np.uint32).astype(np.uint16))
    for up_bits in (0x3F80, 0x3F9E, 0xC000, 0x0001):
        up = np.full_like(gate, O.bf16_from_bits(np.array([up_bits], np.uint16))[0])
        with np.errstate(all="ignore"):
            ref = O.silu_mul_bf16(gate, up)
        out = vxmoe.swiglu(bf16_t(gate), bf16_t(up))
        got = O.bf16_bits(np32(out))
        exp = O.bf16_bits(ref)
        nan = np.isnan(ref)
        assert np.all(np.isnan(np32(out))[nan])
        np.testing.assert_array_equal(got[~nan], exp[~nan])


def test_gather_qmm_matches_qmv_formula(small_params):
    import vxmoe
    p = small_params
    rng = np.random.default_rng(1)
    for T, k in ((1, 1), (3, 4), (37, 4)):
        x = O.make_x(T, T, p.hidden)
        inds = rng.integers(0, p.num_experts, size=(T, k)).astype(np.int32)
        out = vxmoe.gather_qmm(bf16_t(x)[:, None, None, :], *bank_t(p.gate),
                               rhs_indices=torch.from_numpy(inds).to(DEV))
        assert tuple(out.shape) == (T, k, 1, p.gate.w.shape[1])
        ref = np.zeros((T, k, p.gate.w.shape[1]), np.float32)
        for t in range(T):
            for s in range(k):
                b = p.gate.expert(inds[t, s])
                ref[t, s] = O.bf16_round(O.qmv(x[t], b.w, b.scales, b.biases).astype(np.float32))
        assert_bf16_close(np32(out[:, :, 0]), ref, what=f"gather_qmm T={T}")


def test_gather_qmm_lhs_indices_and_slot_inputs(small_params):
    """The down-projection form: x [T, k, 1, I] with per-slot inputs, and an
    explicit lhs index (sorted path of _gather_sort)."""
    import vxmoe
    p = small_params
    rng = np.random.default_rng(2)
    T, k, I = 5, 4, p.down.w.shape[2] * 8
    h = O.bf16_round(rng.normal(0, 0.1, size=(T, k, 1, I)))
    inds = rng.integers(0, p.num_experts, size=(T, k)).astype(np.int32)
    out = vxmoe.gather_qmm(bf16_t(h), *bank_t(p.down), rhs_indices=torch.from_numpy(inds).to(DEV))
    ref = np.zeros((T, k, p.hidden), np.float32)
    for t in range(T):
        for s in range(k):
            b = p.down.expert(inds[t, s])
            ref[t, s] = O.bf16_round(O.qmv(h[t, s, 0], b.w, b.scales, b.biases).astype(np.float32))
    assert_bf16_close(np32(out[:, :, 0]), ref, what="down gather_qmm")
    # sorted form: x_sorted [P, 1, I] gathered with lhs = order // k
    order, inv, sorted_e, _ = O.gather_sort(inds, p.num_experts)
    xs = bf16_t(h.reshape(T * k, 1, I))
    out2 = vxmoe.gather_qmm(xs, *bank_t(p.down), lhs_indices=torch.from_numpy(order).to(DEV),
                            rhs_indices=torch.from_numpy(sorted_e).to(DEV), sorted_indices=True)
    np.testing.assert_array_equal(O.bf16_bits(np32(out2[:, 0])),
                                  O.bf16_bits(np32(out[:, :, 0]).reshape(T * k, -1)[order]))


@pytest.mark.parametrize("K,N", [(32, 8), (96, 24), (160, 40), (2560, 640), (640, 2560)])
def test_gather_qmm_ragged_widths(K, N):
    """Odd group counts, widths that are not a multiple of 128 and row counts
    that are not a multiple of 16 (the Qwen production shape 2560/640 too)."""
    import vxmoe
    rng = np.random.default_rng(K + N)
    bank = O.make_q4_bank(rng, 3, N, K)
    T = 7
    x = O.make_x(K, T, K)
    inds = rng.integers(0, 3, size=(T, 2)).astype(np.int32)
    out = vxmoe.gather_qmm(bf16_t(x)[:, None, None, :], *bank_t(bank),
                           rhs_indices=torch.from_numpy(inds).to(DEV))
    ref = np.stack([np.stack([O.bf16_round(O.qmv(x[t], bank.w[e], bank.scales[e], bank.biases[e])
                                            .astype(np.float32)) for e in inds[t]]) for t in range(T)])
    assert_bf16_close(np32(out[:, :, 0]), ref, what=f"gather_qmm K={K} N={N}")


def test_gather_qmm_many_tokens_per_expert(small_params):
    """An expert with more tokens than one work item holds (items chunked)."""
    import vxmoe
    p = small_params
    T = 50
    x = O.make_x(77, T, p.hidden)
    inds = np.zeros((T, 1), np.int32)
    inds[::3] = 5
    out = vxmoe.gather_qmm(bf16_t(x)[:, None, None, :], *bank_t(p.up),
                           rhs_indices=torch.from_numpy(inds).to(DEV))
    ref = np.stack([O.bf16_round(O.qmv(x[t], p.up.w[inds[t, 0]], p.up.scales[inds[t, 0]],
                                       p.up.biases[inds[t, 0]]).astype(np.float32)) for t in range(T)])
    assert_bf16_close(np32(out[:, 0, 0]), ref, what="many tokens per expert")


def test_gather_qmm_production_width(prod_params):
    import vxmoe
    p = prod_params
    x = O.make_x(3, 2, 2048)
    inds = np.array([[0, 511, 7], [300, 300, 1]], np.int32)
    out = vxmoe.gather_qmm(bf16_t(x)[:, None, None, :], *bank_t(p.up),
                           rhs_indices=torch.from_numpy(inds).to(DEV))
    ref = np.stack([np.stack([O.bf16_round(O.qmv(x[t], p.up.w[e], p.up.scales[e], p.up.biases[e])
                                            .astype(np.float32)) for e in inds[t]]) for t in range(2)])
    assert_bf16_close(np32(out[:, :, 0]), ref, what="production gather_qmm")


# ---------------------------------------------------------------- router

def test_softmax_topk_bit_exact_ids_with_ties():
    import vxmoe
    rng = np.random.default_rng(3)
    T, E, k = 200, 512, 10
    logits = O.bf16_round(rng.normal(0, 1, size=(T, E)))
    # force ties at the selection boundary in some rows
    logits[:20, :40] = O.bf16_round(np.float32(3.0))
    logits[20:30] = O.bf16_round(np.float32(0.5))
    out = vxmoe.softmax_topk(bf16_t(logits), k)
    ref = O.router(None, None, k, logits=logits)
    np.testing.assert_array_equal(out.inds.cpu().numpy(), ref.inds)
    assert ulp_diff_bf16(np32(out.scores), ref.scores).max() <= 1
    assert ulp_diff_bf16(np32(out.weights), ref.weights).max() <= 2
    assert ulp_diff_bf16(np32(out.mass), ref.mass[:, 0]).max() <= 1


@pytest.mark.parametrize("E,k", [(8, 1), (64, 8), (160, 10), (1024, 16)])
def test_softmax_topk_shapes(E, k):
    import vxmoe
    rng = np.random.default_rng(E)
    logits = O.bf16_round(rng.normal(0, 2, size=(33, E)))
    out = vxmoe.softmax_topk(bf16_t(logits), k)
    ref = O.router(None, None, k, logits=logits)
    np.testing.assert_array_equal(out.inds.cpu().numpy(), ref.inds)


def test_router_bias_skews_routing(prod_params):
    """A bf16 logit bias (the skewed-load configuration's +2.0 on 32 hot
    experts) is added to the bf16 logits before softmax/top-k: logits within
    one ulp of the biased float64 oracle, ids bit-exact against the oracle on
    the device's own logits, and most slots go to the hot experts."""
    import vxmoe
    p = prod_params
    w = weights_from_oracle(p)
    rng = np.random.default_rng(3)
    hot = rng.choice(512, 32, replace=False)
    bias = np.zeros(512, np.float32)
    bias[hot] = 2.0
    w.router_bias = torch.from_numpy(bias).to(torch.bfloat16).to(DEV)
    x = O.make_x(6, 32, 2048)
    r = vxmoe.router(bf16_t(x), w)
    ref = O.router(x, p.router_w, 10, bias=bias)
    assert_bf16_close(np32(r.logits), ref.logits, min_exact=0.99, what="biased router logits")
    own = O.router(None, None, 10, logits=np32(r.logits))
    np.testing.assert_array_equal(r.inds.cpu().numpy(), own.inds)
    assert np.isin(r.inds.cpu().numpy(), hot).mean() > 0.5
    y = vxmoe.moe_block(bf16_t(x), w)      # the block takes the same routes
    _, inds, _ = vxmoe.moe_block(bf16_t(x), w, return_routing=True)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(inds.cpu().numpy(), r.inds.cpu().numpy())
    assert torch.isfinite(y.float()).all()


def test_router_full_production(prod_params):
    """Device logits within one bf16 ulp of the float64 oracle; ids bit-exact
    against the oracle run on the device's own logits, and equal to the
    oracle's ids except where the oracle's logits tie across the cut."""
    import vxmoe
    p = prod_params
    w = weights_from_oracle(p)
    x = O.make_x(5, 64, 2048)
    r = vxmoe.router(bf16_t(x), w)
    ref_logits = O.router_logits(x, p.router_w)
    assert_bf16_close(np32(r.logits), ref_logits, min_exact=0.99, what="router logits")
    own = O.router(None, None, 10, logits=np32(r.logits))
    np.testing.assert_array_equal(r.inds.cpu().numpy(), own.inds)
    assert ulp_diff_bf16(np32(r.weights), own.weights).max() <= 2
    ref = O.router(x, p.router_w, 10)
    for t in range(64):
        if set(r.inds[t].tolist()) != set(ref.inds[t].tolist()):
            srt = np.sort(ref.logits[t])[::-1]
            assert ulp_diff_bf16(srt[9:10], srt[10:11]).max() <= 1, f"row {t} differs without a near-tie"
    # shared expert gate
    seg = p.shared_expert_gate.expert(0)
    z = O.bf16_round(O.qmv(x, seg.w, seg.scales, seg.biases).astype(np.float32))
    assert ulp_diff_bf16(np32(r.shared_gate), O.sigmoid_bf16(z)).max() <= 1


@pytest.mark.parametrize("biased", [False, True])
def test_router_tiled_prefill_equals_fused(prod_params, biased):
    """Batches of 256 tokens or more take the tiled logits kernel and the
    separate softmax/top-k kernel; smaller ones the fused single launch.  The
    two sum the logits in the same order, so a 600-token batch must give the
    bits of the same tokens routed in 200-token pieces: logits, ids, weights
    and the shared-expert gate."""
    import vxmoe
    p = prod_params
    w = weights_from_oracle(p)
    if biased:
        bias = np.zeros(512, np.float32)
        bias[np.random.default_rng(4).choice(512, 32, replace=False)] = 2.0
        w.router_bias = torch.from_numpy(bias).to(torch.bfloat16).to(DEV)
    x = bf16_t(O.make_x(8, 600, 2048))
    whole = vxmoe.router(x, w)
    parts = [vxmoe.router(x[a:a + 200], w) for a in (0, 200, 400)]
    torch.cuda.synchronize()
    for name in ("logits", "inds", "weights", "shared_gate"):
        got = getattr(whole, name)
        exp = torch.cat([getattr(r, name) for r in parts])
        np.testing.assert_array_equal(got.view(torch.int16).cpu().numpy() if got.dtype == torch.bfloat16
                                      else got.cpu().numpy(),
                                      exp.view(torch.int16).cpu().numpy() if exp.dtype == torch.bfloat16
                                      else exp.cpu().numpy(), err_msg=name)


# ---------------------------------------------------------------- permutation

@pytest.mark.parametrize("P,E,skew", [(0, 8, False), (1, 8, False), (10, 512, False),
                                      (200, 512, False), (256, 1024, False), (256, 8, True),
                                      (257, 512, True), (80, 3, False),
                                      (640, 512, False), (1024, 1024, True), (1024, 8, False),
                                      (513, 1, False), (1025, 512, True),
                                      (4096, 64, True), (65536, 512, True),
                                      (20480, 512, False), (100003, 64, False)])
def test_permute_bit_exact(P, E, skew):
    import vxmoe
    rng = np.random.default_rng(P + E)
    if skew:
        ids = np.where(rng.random(P) < 0.7, rng.integers(0, 4, P), rng.integers(0, E, P))
    else:
        ids = rng.integers(0, E, P)
    ids = ids.astype(np.int32)
    perm = vxmoe.permute(torch.from_numpy(ids).to(DEV), E)
    order, inv, _, offsets = O.gather_sort(ids, E)
    np.testing.assert_array_equal(perm.order.cpu().numpy(), order)
    np.testing.assert_array_equal(perm.inverse.cpu().numpy(), inv)
    np.testing.assert_array_equal(perm.offsets.cpu().numpy(), offsets)
    assert int(perm.errors.item()) == 0


@pytest.mark.parametrize("P", [40000, 900])
def test_permute_large_drops_out_of_range_ids(P):
    """Prefill-sized input (the multi-CTA permutation) and a decode-sized one
    (the one-CTA permutation, four ids a thread): invalid ids are counted,
    get inverse -1 and leave the order of the others stable."""
    import vxmoe
    rng = np.random.default_rng(77)
    ids = rng.integers(0, 256, P).astype(np.int32)
    bad = rng.random(P) < 0.01
    ids[bad] = np.where(rng.random(int(bad.sum())) < 0.5, -1, 256)
    perm = vxmoe.permute(torch.from_numpy(ids).to(DEV), 256)
    good = np.nonzero(~bad)[0]
    order = good[np.argsort(ids[good], kind="stable")]
    np.testing.assert_array_equal(perm.order.cpu().numpy()[:good.size], order)
    inv = perm.inverse.cpu().numpy()
    assert (inv[bad] == -1).all()
    np.testing.assert_array_equal(inv[order], np.arange(good.size))
    assert int(perm.errors.item()) == int(bad.sum())


def test_permute_counts_out_of_range_ids():
    import vxmoe
    ids = np.array([3, -1, 9, 2, 3], np.int32)
    perm = vxmoe.permute(torch.from_numpy(ids).to(DEV), 4)
    assert int(perm.errors.item()) == 2
    assert perm.offsets.cpu().numpy().tolist() == [0, 0, 0, 1, 3]
    inv = perm.inverse.cpu().numpy()
    assert inv[1] == -1 and inv[2] == -1
    np.testing.assert_array_equal(perm.order.cpu().numpy()[:3], [3, 0, 4])


# ---------------------------------------------------------------- executor and block

def _executor_ref(p, x, routes, scores, shared_y=None):
    yd = np.zeros((x.shape[0], routes.shape[1], p.hidden), np.float32)
    for t in range(x.shape[0]):
        for s in range(routes.shape[1]):
            e = routes[t, s]
            yd[t, s] = O.expert_mlp_bf16(x[t:t + 1], p.gate.expert(e), p.up.expert(e),
                                         p.down.expert(e))[3][0]
    if scores is None:
        return yd
    return O.fused_combine(yd, scores, shared_y)


def test_executor_per_slot_and_combined(small_params):
    import vxmoe
    p = small_params
    rng = np.random.default_rng(4)
    T, k = 6, 4
    x = O.make_x(9, T, p.hidden)
    routes = rng.integers(0, p.num_experts, size=(T, k)).astype(np.int32)
    routes[0, 1] = routes[0, 0]          # a token routed twice to one expert
    scores = O.bf16_round(rng.random((T, k)).astype(np.float32) / k)
    shared_y = O.bf16_round(rng.normal(0, 0.01, size=(T, p.hidden)))
    ex = vxmoe.build_executor(expert_count=p.num_experts, hidden_size=p.hidden, top_k=k)
    packs = {"gate_proj": bank_t(p.gate), "up_proj": bank_t(p.up), "down_proj": bank_t(p.down)}
    xt, rt = bf16_t(x), torch.from_numpy(routes).to(DEV)
    per_slot = ex.execute(xt, rt, packs)
    assert ex.last_path == "custom-cuda"
    ref_slot = _executor_ref(p, x, routes, None)
    assert O.normwise_error(np32(per_slot), ref_slot) < 1e-2
    assert float(np.mean(ulp_diff_bf16(np32(per_slot), ref_slot) == 0)) > 0.9
    comb = ex.execute(xt, rt, packs, scores=bf16_t(scores), shared_y=bf16_t(shared_y))
    ref = _executor_ref(p, x, routes, scores, shared_y)
    assert O.normwise_error(np32(comb), ref) < 1e-2
    # same bf16 slot outputs in -> bit-exact combine
    exact = O.fused_combine(np32(per_slot), scores, shared_y)
    np.testing.assert_array_equal(O.bf16_bits(np32(comb)), O.bf16_bits(exact))
    # shared parts form equals shared_y = bf16(sg * shared)
    shared = O.bf16_round(rng.normal(0, 0.05, size=(T, p.hidden)))
    sg = O.bf16_round(rng.random((T, 1)).astype(np.float32))
    parts = ex.execute(xt, rt, packs, scores=bf16_t(scores), shared=bf16_t(shared),
                       shared_gate=bf16_t(sg))
    exact2 = O.fused_combine(np32(per_slot), scores, O.bf16_round(sg * shared))
    np.testing.assert_array_equal(O.bf16_bits(np32(parts)), O.bf16_bits(exact2))
    g, u, d = ex.execute(xt, rt, packs, return_all=True)
    assert tuple(g.shape) == (T, k, 64) and tuple(d.shape) == (T, k, p.hidden)


def test_executor_against_reference_golden(golden_dir):
    """The reference executor's own outputs (float32 NumPy path, float32
    SiLU) within the tolerance of the reference's custom-vs-gather_qmm test
    (test_metal_runtime.py:321-350)."""
    import vxmoe
    g = np.load(os.path.join(golden_dir, "executor.npz"))
    packs = {n: (u32_t(g[f"{n[:-5]}_w"]), bf16_t(g[f"{n[:-5]}_s"]), bf16_t(g[f"{n[:-5]}_b"]))
             for n in ("gate_proj", "up_proj", "down_proj")}
    T, D = g["x"].shape
    ex = vxmoe.build_executor(expert_count=4, hidden_size=D, top_k=2)
    xt, rt = bf16_t(g["x"]), torch.from_numpy(g["routes"]).to(DEV)
    gate, up, down = ex.execute(xt, rt, packs, return_all=True)
    np.testing.assert_allclose(np32(gate), g["gate_out"], rtol=2e-2, atol=3e-3)
    np.testing.assert_allclose(np32(up), g["up_out"], rtol=2e-2, atol=3e-3)
    np.testing.assert_allclose(np32(down), g["down_out"], rtol=2e-2, atol=3e-3)
    comb = ex.execute(xt, rt, packs, scores=bf16_t(g["scores"]))
    np.testing.assert_allclose(np32(comb), g["combined"], rtol=2e-2, atol=3e-3)


def _block_check(p, x, what):
    """The block against the oracle on the device's logits, with the oracle's
    expert arithmetic matching the device path the batch takes (the tcgen05
    GEMM's bf16-dequantised tiles once T*k >= 4E, MLX's qmv below)."""
    import vxmoe
    w = weights_from_oracle(p)
    y, inds, wts = vxmoe.moe_block(bf16_t(x), w, return_routing=True)
    logits = np32(vxmoe.router(bf16_t(x), w).logits)
    path = "prefill" if x.shape[0] * p.top_k >= 4 * p.num_experts else "decode"
    out = O.moe_block(x, p, logits=logits, path=path)
    np.testing.assert_array_equal(inds.cpu().numpy(), out.router.inds)
    got = np32(y)
    ref = O.moe_block_reference_f64(x, p, out.router.inds, out.router.logits)
    scale = O.summand_scale(out.yd, out.router.weights, out.shared_y)
    assert_block_bar(got, out.y, ref, scale, f"{what} ({path})")
    rms = np.linalg.norm(got - ref) / np.linalg.norm(ref)
    assert rms < 1e-2, f"{what}: rms vs float64 {rms}"
    return got, out


def test_block_small_shapes(small_params):
    for T in (1, 2, 8, 33):
        _block_check(small_params, O.make_x(20 + T, T, small_params.hidden), f"small T={T}")


def test_block_production_decode(prod_params):
    for T in (1, 8):
        _block_check(prod_params, O.make_x(1, T, 2048), f"production T={T}")


@pytest.mark.slow
def test_block_production_batched_decode(prod_params):
    _block_check(prod_params, O.make_x(1, 64, 2048), "production T=64")


def test_block_production_fused_permutation_many_token_blocks(prod_params):
    """T*k = 1000 routes: the last of 13 token blocks of the fused router
    sorts them (second arrival), four ids a thread."""
    _block_check(prod_params, O.make_x(5, 100, 2048), "production T=100")


def test_block_empty_batch(small_params):
    import vxmoe
    w = weights_from_oracle(small_params)
    y = vxmoe.moe_block(torch.empty((0, small_params.hidden), dtype=torch.bfloat16, device=DEV), w)
    assert tuple(y.shape) == (0, small_params.hidden)


def test_block_without_shared_expert(small_params):
    import vxmoe
    p = small_params
    w = weights_from_oracle(p, shared=False)
    x = O.make_x(3, 4, p.hidden)
    y = vxmoe.moe_block(bf16_t(x), w)
    r = O.router(x, p.router_w, p.top_k, logits=np32(vxmoe.router(bf16_t(x), w).logits))
    yd, _ = O.routed_outputs(x, r.inds, p)
    ref = O.fused_combine(yd, r.weights, None)
    assert O.normwise_error(np32(y), ref) < 1e-2


def test_rmsnorm_matches_oracle():
    import vxmoe
    rng = np.random.default_rng(8)
    x = O.bf16_round(rng.normal(0, 1, size=(16, 2048)))
    gain = O.bf16_round(np.ones(2048, np.float32))
    y = vxmoe.rms_norm(bf16_t(x), bf16_t(gain), 1e-6)
    assert ulp_diff_bf16(np32(y), O.rms_norm(x, gain, 1e-6)).max() <= 1


def test_errors_raise_reference_exception_types(small_params):
    import vxmoe
    p = small_params
    with pytest.raises(TypeError):
        vxmoe.gather_qmm(bf16_t(np.zeros((1, 1, p.hidden), np.float32)),
                         torch.zeros((2, 4, p.hidden // 8), dtype=torch.int32, device=DEV),
                         bf16_t(np.zeros((2, 4, p.hidden // 32))), bf16_t(np.zeros((2, 4, p.hidden // 32))),
                         rhs_indices=torch.zeros((1,), dtype=torch.int32, device=DEV))
    with pytest.raises(ValueError):
        vxmoe.gather_qmm(bf16_t(np.zeros((1, 1, 64), np.float32)), *bank_t(p.gate),
                         rhs_indices=torch.zeros((1,), dtype=torch.int32, device=DEV))
    with pytest.raises(ValueError):
        vxmoe.gather_qmm(bf16_t(np.zeros((1, 1, p.hidden), np.float32)), *bank_t(p.gate),
                         rhs_indices=np.array([40], np.int32))


def test_weighted_combine_on_the_device(golden_dir):
    """The executor's combine-only form on CUDA tensors runs the library's
    combine kernel: the reference helper's unit values (float32), and bf16
    slot and all-expert forms against the array expression it replaces."""
    import vxmoe
    g = np.load(os.path.join(golden_dir, "combine.npz"))
    f32 = lambda a: torch.from_numpy(np.ascontiguousarray(np.asarray(a, np.float32))).to(DEV)
    got = vxmoe.weighted_combine(f32(g["eo2"]), torch.from_numpy(g["r2"]).to(DEV), f32(g["sc2"]))
    np.testing.assert_array_equal(got.cpu().numpy(), g["c2"])
    got = vxmoe.weighted_combine(f32(g["slot"]), torch.from_numpy(g["r3"]).to(DEV), f32(g["sc3"]))
    np.testing.assert_array_equal(got.cpu().numpy(), g["c3"])
    gen = torch.Generator(device=DEV)
    gen.manual_seed(3)
    T, k, E, d = 37, 10, 24, 2048
    out = torch.randn((T, E, d), device=DEV, generator=gen).to(torch.bfloat16)
    routes = torch.stack([torch.randperm(E, device=DEV, generator=gen)[:k] for _ in range(T)]).int()
    scores = torch.rand((T, k), device=DEV, generator=gen).to(torch.bfloat16)
    y = vxmoe.weighted_combine(out, routes, scores)
    sel = torch.take_along_dim(out, routes[..., None].long(), dim=-2)
    ref = (sel.float() * scores.float()[..., None]).to(torch.bfloat16).float().sum(-2)   # bf16 products
    assert ulp_diff_bf16(np32(y), np32(ref.to(torch.bfloat16))).max() <= 1
    y_slot = vxmoe.weighted_combine(sel.contiguous(), routes, scores)
    assert torch.equal(y_slot.view(torch.int16), y.view(torch.int16))
    with pytest.raises(ValueError):
        vxmoe.weighted_combine(out, routes + E, scores)
