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
