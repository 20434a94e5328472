"""Shared helpers of the GPU tests: move oracle arrays onto the device and
back, and the comparison rules used throughout."""
from __future__ import annotations

import numpy as np
import torch

import vxmoe_oracle as O


def bf16_t(a, device="cuda") -> torch.Tensor:
    """float32 array of bf16 values -> bf16 CUDA tensor (exact)."""
    return torch.from_numpy(np.ascontiguousarray(np.asarray(a, dtype=np.float32))).to(
        device=device, dtype=torch.bfloat16)


def u32_t(a, device="cuda") -> torch.Tensor:
    return torch.from_numpy(np.ascontiguousarray(a)).to(device)


def np32(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


def bank_t(b: "O.Q4Bank", device="cuda"):
    return (u32_t(b.w, device), bf16_t(b.scales, device), bf16_t(b.biases, device))


def weights_from_oracle(p: "O.MoEParams", device="cuda", shared=True):
    import vxmoe
    kw = {}
    if shared:
        kw = dict(shared_gate=bank_t(p.shared_gate, device), shared_up=bank_t(p.shared_up, device),
                  shared_down=bank_t(p.shared_down, device),
                  shared_expert_gate=bank_t(p.shared_expert_gate, device))
    return vxmoe.MoEWeights(bank_t(p.gate, device), bank_t(p.up, device), bank_t(p.down, device),
                            router_w=bf16_t(p.router_w, device), top_k=p.top_k, device=device, **kw)


def ulp_diff_bf16(a, b) -> np.ndarray:
    """Distance in bf16 ulps between two arrays of bf16 values (same sign
    convention as the integer encoding)."""
    ia = O.bf16_bits(a).astype(np.int32)
    ib = O.bf16_bits(b).astype(np.int32)
    ia = np.where(ia & 0x8000, 0x8000 - ia, ia)
    ib = np.where(ib & 0x8000, 0x8000 - ib, ib)
    return np.abs(ia - ib)


def assert_bf16_close(actual, expected, max_ulp=1, min_exact=0.97, floor=2.0 ** -12, what=""):
    """bf16 outputs of float accumulations: the device sums in float32, the
    oracle in float64, so a value may land one bf16 ulp away when the exact
    sum is near a rounding boundary.  Values whose magnitude is below
    `floor` x rms(expected) (sums that cancel to nearly zero, where one bf16
    ulp is a tiny fraction of the data's scale) may instead differ by at most
    `floor` x rms in absolute terms.  Nothing else may be further off."""
    a = np.asarray(actual, dtype=np.float64)
    r = np.asarray(expected, dtype=np.float64)
    d = ulp_diff_bf16(actual, expected)
    exact = float(np.mean(d == 0)) if d.size else 1.0
    scale = float(np.sqrt(np.mean(r * r))) if r.size else 0.0
    ok = (d <= max_ulp) | (np.abs(a - r) <= floor * scale)
    assert ok.all(), f"{what}: max ulp diff {d[~ok].max()} at |ref|={np.abs(r[~ok]).min():.3g} (rms {scale:.3g})"
    assert exact >= min_exact, f"{what}: only {exact:.4f} exact"


def block_errors(got, oracle_y, ref64, scale):
    """Errors of a block output against the bf16-semantics oracle and the
    unrounded float64 reference.  max_rel_*: max |a-r| / max(|r|, scale),
    the denominator floored per output by `scale`, the magnitude of the terms
    the output sums (oracle.summand_scale: sum_s |w_s y_s| + |shared_y|) - an
    output that cancels to near zero is measured against its summands;
    max_rel_rms_*: the same with the floor at the output's rms (reported
    only); normwise_*: max abs error over max |ref|; allclose_*: the
    reference harness's allclose(atol=rtol=1e-2)
    (models/flashnext/tests/bench/bench_runtime_layer.py:471-472)."""
    got = np.asarray(got, dtype=np.float64)
    out = {}
    for name, ref in (("oracle", oracle_y), ("f64", ref64)):
        ref = np.asarray(ref, dtype=np.float64)
        out[f"max_rel_{name}"] = O.max_rel_error_floored(got, ref, scale)
        out[f"max_rel_rms_{name}"] = O.max_rel_error(got, ref, 1.0)
        out[f"normwise_{name}"] = O.normwise_error(got, ref)
        out[f"allclose_{name}"] = bool(np.allclose(got, ref, atol=1e-2, rtol=1e-2))
    ref64 = np.asarray(ref64, dtype=np.float64)
    out["max_rel_oracle_own_f64"] = O.max_rel_error_floored(oracle_y, ref64, scale)
    out["normwise_oracle_own_f64"] = O.normwise_error(oracle_y, ref64)
    return out


def assert_block_bar(got, oracle_y, ref64, scale, what):
    """The block-output bar, printed and asserted:
    * against the oracle (the reference's bf16 arithmetic restated): max
      relative error <= 1e-2 with the summand-magnitude floor, and normwise
      error < 1e-2;
    * against the float64 reference: no worse than the reference's own bf16
      arithmetic (the oracle) by more than 25 % + 2e-3, in both metrics - the
      oracle itself sits at 1-3e-2 max relative error from exact math, so a
      literal 1e-2 there would reject the reference's own arithmetic;
    * allclose(atol=rtol=1e-2) against both, the reference harness's check."""
    e = block_errors(got, oracle_y, ref64, scale)
    print(f"[block bar] {what}: " + ", ".join(
        f"{k}={v:.3e}" if isinstance(v, float) else f"{k}={v}" for k, v in e.items()))
    assert e["max_rel_oracle"] <= 1e-2, f"{what}: floored max rel error vs oracle {e['max_rel_oracle']}"
    assert e["normwise_oracle"] < 1e-2, f"{what}: normwise error vs oracle {e['normwise_oracle']}"
    assert e["max_rel_f64"] <= 1.25 * e["max_rel_oracle_own_f64"] + 2e-3, \
        f"{what}: max rel vs f64 {e['max_rel_f64']} (oracle's own {e['max_rel_oracle_own_f64']})"
    assert e["normwise_f64"] <= 1.25 * e["normwise_oracle_own_f64"] + 2e-3, \
        f"{what}: normwise vs f64 {e['normwise_f64']} (oracle's own {e['normwise_oracle_own_f64']})"
    assert e["allclose_oracle"] and e["allclose_f64"], f"{what}: allclose(1e-2, 1e-2) failed"
    return e


def assert_same_products(a, b, what, min_identical=0.95, max_normwise=1e-2):
    """Two GPU paths that form the same exact products q * x and differ only
    in the float32 order (or scale) of their sums: a g or u value may round
    one bf16 ulp apart, and through h and the down projection that moves an
    output by up to ~1e-2 of the rms (many of its own ulps when it cancels to
    near zero).  Most outputs keep their bits; each path's bar against the
    oracle is checked on its own."""
    a, b = np32(a), np32(b)
    exact = float(np.mean(O.bf16_bits(a) == O.bf16_bits(b)))
    err = O.normwise_error(a, b)
    assert exact >= min_identical and err < max_normwise, \
        f"{what}: {exact:.4f} identical, normwise {err:.2e}"
