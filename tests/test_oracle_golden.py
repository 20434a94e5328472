"""Pin the CPU oracle to the reference's own NumPy code (golden fixtures) and
to the known-answer values of the reference's unit tests."""
from __future__ import annotations

import os

import numpy as np
import pytest

import vxmoe_oracle as O


def _load(golden_dir, name):
    return np.load(os.path.join(golden_dir, name))


def test_nibble_unpack_and_dequant_match_reference(golden_dir):
    g = _load(golden_dir, "dequant.npz")
    deq = O.dequantize(g["w"], g["scales"], g["biases"])
    np.testing.assert_array_equal(deq.view(np.uint32), g["dequant"].view(np.uint32))
    q = O.q4_unpack(g["w"])
    assert q.shape == (2, 4, 64)
    np.testing.assert_array_equal(O.q4_pack(q), g["w"])


def test_unpack_bit_layout_low_nibble_first():
    w = np.array([[0x76543210, 0xFEDCBA98]], dtype=np.uint32)
    np.testing.assert_array_equal(O.q4_unpack(w)[0], np.arange(16))


def test_unpack_rejects_non_uint32():
    with pytest.raises(TypeError):
        O.q4_unpack(np.zeros((2, 2), dtype=np.int32))


def test_projection_matches_reference_numpy_path(golden_dir):
    g = _load(golden_dir, "projection.npz")
    out = O.numpy_projection(g["x"], g["routes"], g["w"], g["scales"], g["biases"],
                             g["w"].shape[1], False)
    np.testing.assert_array_equal(out, g["out"])


def test_executor_reference_path_matches(golden_dir):
    g = _load(golden_dir, "executor.npz")
    bank = lambda p: O.Q4Bank(g[p + "_w"], g[p + "_s"], g[p + "_b"])
    gate, up, down = bank("gate"), bank("up"), bank("down")
    go, uo, do = O.executor_reference_all(g["x"], g["routes"], gate, up, down,
                                          hidden_size=g["x"].shape[1])
    np.testing.assert_array_equal(go, g["gate_out"])
    np.testing.assert_array_equal(uo, g["up_out"])
    np.testing.assert_array_equal(do, g["down_out"])
    comb = O.weighted_combine(do, g["routes"], g["scores"])
    np.testing.assert_array_equal(comb, g["combined"])


def test_weighted_combine_known_answers(golden_dir):
    g = _load(golden_dir, "combine.npz")
    c1 = O.weighted_combine(g["eo"], g["r"], g["sc"])
    np.testing.assert_array_equal(c1, np.array([[25.75, 51.5], [192.0, 256.0]], np.float32))
    np.testing.assert_array_equal(c1, g["c1"])
    np.testing.assert_array_equal(O.weighted_combine(g["eo2"], g["r2"], g["sc2"]), g["c2"])
    np.testing.assert_array_equal(O.weighted_combine(g["slot"], g["r3"], g["sc3"]), g["c3"])


def test_weighted_combine_rejects_bad_routes():
    eo = np.zeros((2, 3, 2), np.float32)
    with pytest.raises(ValueError):
        O.weighted_combine(eo, np.zeros((2, 2), np.int32), np.ones((2, 1), np.float32))
    with pytest.raises(ValueError):
        O.weighted_combine(eo, np.array([[0, 3]], np.int32), np.ones((1, 2), np.float32))


def test_bf16_round_trip_and_rne():
    raw = np.array([0x0000, 0x3F80, 0x8000, 0x7F80, 0xFFFF], dtype=np.uint16)
    v = O.bf16_from_bits(raw)
    out = O.bf16_bits(v)
    np.testing.assert_array_equal(out[:4], raw[:4])
    assert np.isnan(v[4])
    # ties to even: 1 + 2^-8 is halfway between 1 and 1+2^-7 -> 1
    assert O.bf16_round(np.float32(1 + 2**-8)) == np.float32(1.0)
    assert O.bf16_round(np.float32(1 + 3 * 2**-8)) == np.float32(1 + 2**-6)


def test_swiglu_representative_values():
    """The reference's representative SwiGLU contract inputs
    (test_swiglu_contract.py:25-31); expected values follow from the bf16
    sequence and are stated here as bit patterns."""
    gate = O.bf16_from_bits([0x0000, 0x3F80, 0xBF80, 0x4120, 0xC120])
    up = O.bf16_from_bits([0x3F80, 0x3FA0, 0x3F00, 0x4020, 0xC000])
    h = O.silu_mul_bf16(gate, up)
    # silu(0)=0; silu(1)=0.7305*1.25; silu(-1)=-0.2695*0.5; silu(10)=9.9995->10*2.5; silu(-10)~-4.5e-4*-2
    assert O.bf16_bits(h)[0] == 0x0000
    ref = np.array([0.0, 0.7310586 * 1.25, -0.26894143 * 0.5, 9.999546 * 2.5, -4.539787e-4 * -2.0])
    np.testing.assert_allclose(h, ref, rtol=2 ** -6)


def test_swiglu_bf16_exhaustive_properties():
    """Exhaustive over every bf16 gate encoding at up=1.0: the bf16 sequence
    stays within a few bf16 ulps of float64 silu, and differs from an fp32
    silu rounded once (as the reference's contract test says it should)."""
    gate = O.bf16_from_bits(np.arange(65536, dtype=np.uint32).astype(np.uint16))
    up = np.ones_like(gate)
    h = O.silu_mul_bf16(gate, up)
    finite = np.isfinite(gate) & (np.abs(gate) < 80)
    g64 = gate.astype(np.float64)
    with np.errstate(all="ignore"):
        exact = g64 / (1 + np.exp(-g64))
        rel = np.abs(h[finite] - exact[finite]) / np.maximum(np.abs(exact[finite]), 1e-30)
        fp32_once = O.bf16_round(exact.astype(np.float32))
    big = np.abs(exact[finite]) > 1e-30
    assert np.max(rel[big]) < 2 ** -4
    assert np.count_nonzero(O.bf16_bits(fp32_once[finite]) != O.bf16_bits(h[finite])) > 0


def test_router_topk_tie_rule_and_renorm():
    logits = O.bf16_round(np.array([[0.5, 1.0, 1.0, -2.0, 1.0, 0.25]], np.float32))
    r = O.router(None, None, 3, logits=logits)
    np.testing.assert_array_equal(r.inds, [[1, 2, 4]])
    assert abs(float(r.weights.sum()) - 1.0) < 2 ** -6
    # the selected set is a valid top-k of the probabilities
    sel = r.probs[0, r.inds[0]]
    rest = np.delete(r.probs[0], r.inds[0])
    assert sel.min() >= rest.max()


def test_gather_sort_is_stable_and_inverts():
    inds = np.array([[3, 1], [1, 3], [0, 3]], np.int32)
    order, inv, sorted_e, offsets = O.gather_sort(inds, 4)
    np.testing.assert_array_equal(order, [4, 1, 2, 0, 3, 5])
    np.testing.assert_array_equal(sorted_e, [0, 1, 1, 3, 3, 3])
    np.testing.assert_array_equal(offsets, [0, 1, 3, 3, 6])
    np.testing.assert_array_equal(order[inv], np.arange(6))


def test_qmv_equals_dequantized_matmul():
    rng = np.random.default_rng(3)
    b = O.make_q4_bank(rng, 1, 16, 256)
    x = O.make_x(4, 5, 256)
    y = O.qmv(x, b.w[0], b.scales[0], b.biases[0])
    dense = O.dequantize(b.w[0], b.scales[0], b.biases[0]).astype(np.float64)
    np.testing.assert_allclose(y, x.astype(np.float64) @ dense.T, rtol=1e-9, atol=1e-9)


def test_block_bf16_semantics_close_to_unrounded_reference():
    p = O.make_params(seed=5, experts=32, hidden=256, inter=64, shared_inter=64, top_k=4)
    x = O.make_x(6, 4, 256)
    out = O.moe_block(x, p)
    ref = O.moe_block_reference_f64(x, p, out.router.inds, out.router.logits)
    rms = np.linalg.norm(out.y - ref) / np.linalg.norm(ref)
    assert rms < 1e-2
    gen = O.moe_block(x, p, semantics="generic")
    assert np.linalg.norm(gen.y - ref) / np.linalg.norm(ref) < 1e-2
