"""Generate the golden vectors that pin the oracle to the reference's own code.

Run in a checkout where the Veystrix-Core reference tree is available:

    python tests/golden/make_golden.py --reference <path-to-Veystrix-Core>

It imports the reference's NumPy executor path, which runs without MLX
(``models/flashnext/metal_runtime.py``: ``MetalMoEExecutor(...,
backend="reference")`` -> ``_reference_all`` -> ``_numpy_projection``,
``:897-909``, ``:976-983``, ``:997-1029``; ``weighted_combine`` ``:145-191``),
and writes small ``.npz`` fixtures next to this script.  The tests read only
the fixtures; nothing at test time touches the reference tree.
"""
from __future__ import annotations

import argparse
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def _bf16(a):
    a = np.ascontiguousarray(np.asarray(a, dtype=np.float32))
    bits = a.view(np.uint32).astype(np.uint64)
    lsb = (bits >> 16) & 1
    return ((bits + 0x7FFF + lsb) & 0xFFFF0000).astype(np.uint32).view(np.float32).reshape(a.shape)


def _bank(rng, experts, out_w, in_w, gs=32, affine="test"):
    w = rng.integers(0, 2**32, size=(experts, out_w, in_w // 8), dtype=np.uint64).astype(np.uint32)
    if affine == "test":
        # The distribution of the reference's own production-shape test
        # (test_metal_runtime.py:178-186): scales ~N(0.08, 0.01),
        # biases ~N(0, 0.01), stored as bf16.
        s = _bf16(rng.normal(0.08, 0.01, size=(experts, out_w, in_w // gs)))
        b = _bf16(rng.normal(0.0, 0.01, size=(experts, out_w, in_w // gs)))
    else:
        s = _bf16(np.abs(rng.normal(0.0, 0.02, size=(experts, out_w, in_w // gs))) / 8)
        b = (np.float32(-8) * s).astype(np.float32)
    return w, s, b


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    args = ap.parse_args(argv)
    sys.path.insert(0, os.path.abspath(args.reference))
    from models.flashnext.metal_runtime import (  # noqa: E402
        MetalMoEExecutor, Q4G32Projection, _numpy_projection, weighted_combine,
    )

    rng = np.random.default_rng(20260901)

    # A. Nibble unpack and dequant: one-hot inputs through _numpy_projection
    #    return the dequantised weights column by column.
    E, OUT, IN = 2, 4, 64
    w, s, b = _bank(rng, E, OUT, IN)
    proj = Q4G32Projection(w, s, b)
    eye = np.eye(IN, dtype=np.float32)
    deq = np.zeros((E, OUT, IN), dtype=np.float32)
    for e in range(E):
        routes = np.full((IN, 1), e, dtype=np.int32)
        out = _numpy_projection(eye, routes, proj, OUT, False, 32)
        deq[e] = out[:, 0, :].T
    np.savez_compressed(os.path.join(HERE, "dequant.npz"), w=w, scales=s, biases=b, dequant=deq)

    # B. Projection with the synthetic benchmark distribution (bias=-8*scale).
    E, OUT, IN, T, K = 3, 8, 128, 3, 2
    w, s, b = _bank(rng, E, OUT, IN, affine="bench")
    x = _bf16(rng.normal(0, 1, size=(T, IN)))
    routes = rng.integers(0, E, size=(T, K)).astype(np.int32)
    out = _numpy_projection(x, routes, Q4G32Projection(w, s, b), OUT, False, 32)
    np.savez_compressed(os.path.join(HERE, "projection.npz"), w=w, scales=s, biases=b,
                        x=x, routes=routes, out=out)

    # C. Executor reference path, return_all and combined with scores.
    E, D, I, T, K = 4, 64, 32, 3, 2
    gate = _bank(rng, E, I, D)
    up = _bank(rng, E, I, D)
    down = _bank(rng, E, D, I)
    x = _bf16(rng.normal(0, 0.1, size=(T, D)))
    routes = np.array([[0, 2], [3, 1], [2, 2]], dtype=np.int32)
    scores = np.array([[0.25, 0.75], [0.6, 0.4], [0.5, 0.5]], dtype=np.float32)
    ex = MetalMoEExecutor(E, D, K, backend="reference", max_width=64)
    projections = {"gate_proj": gate, "up_proj": up, "down_proj": down}
    g_out, u_out, d_out = ex.execute(x, routes, projections, return_all=True)
    combined = ex.execute(x, routes, projections, scores=scores)
    assert ex.last_path == "reference"
    np.savez_compressed(
        os.path.join(HERE, "executor.npz"),
        gate_w=gate[0], gate_s=gate[1], gate_b=gate[2],
        up_w=up[0], up_s=up[1], up_b=up[2],
        down_w=down[0], down_s=down[1], down_b=down[2],
        x=x, routes=routes, scores=scores,
        gate_out=g_out, up_out=u_out, down_out=d_out, combined=combined)

    # D. weighted_combine: the unit-test values (test_metal_runtime.py:221-238)
    #    and a random case in both the slot form and the all-experts form.
    eo = np.array([[[1.0, 2.0], [10.0, 20.0], [100.0, 200.0]],
                   [[3.0, 4.0], [30.0, 40.0], [300.0, 400.0]]], dtype=np.float32)
    r = np.array([[2, 0], [1, 2]], dtype=np.int32)
    sc = np.array([[0.25, 0.75], [0.4, 0.6]], dtype=np.float32)
    c1 = weighted_combine(eo, r, sc)
    eo2 = rng.normal(size=(5, 7, 16)).astype(np.float32)
    r2 = rng.integers(0, 7, size=(5, 3)).astype(np.int32)
    sc2 = rng.random(size=(5, 3)).astype(np.float32)
    c2 = weighted_combine(eo2, r2, sc2)
    slot = rng.normal(size=(4, 3, 8)).astype(np.float32)
    r3 = np.zeros((4, 3), dtype=np.int32)
    sc3 = rng.random(size=(4, 3)).astype(np.float32)
    c3 = weighted_combine(slot, r3, sc3)
    np.savez_compressed(os.path.join(HERE, "combine.npz"), eo=eo, r=r, sc=sc, c1=c1,
                        eo2=eo2, r2=r2, sc2=sc2, c2=c2, slot=slot, r3=r3, sc3=sc3, c3=c3)
    print("wrote fixtures to", HERE)


if __name__ == "__main__":
    main()
