"""Golden keep counts of adaptive top-k from the reference's own keep rule.

Run in a checkout where the Veystrix-Core reference tree is available:

    python tests/golden/make_adaptive_golden.py --reference <path-to-Veystrix-Core>

It imports models/flashnext/adaptive_topk.py and calls its `_keep_for_mass`
(:44-51) - the Python loop the block runs over each token's top-k weights
(:107-118) - on weight rows of the block's kind: the renormalised top-10 of a
softmax over 512 bf16 logits, bf16-rounded and in descending order, plus rows
that tie, hit a threshold exactly or hold zeros.  The module also imports MLX
and three runtime modules at the top, which the keep rule never calls; they
are replaced by empty stand-ins for the import.  The counts are written to
adaptive_keep.npz beside this script; nothing at test time touches the
reference tree.
"""
from __future__ import annotations

import argparse
import os
import sys
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
THRESHOLDS = [0.0, 0.1, 0.25, 0.5, 0.6, 0.7, 0.75, 0.8, 0.9, 0.95, 0.99, 1.0, 1.5]


def weight_rows():
    sys.path.insert(0, os.path.join(HERE, "..", "..", "oracle"))
    import vxmoe_oracle as O
    rng = np.random.default_rng(20261202)
    rows = []
    for scale in (0.5, 1.0, 2.0, 4.0):
        logits = O.bf16_round(rng.standard_normal((60, 512)).astype(np.float32) * scale)
        p = np.exp(logits - logits.max(axis=1, keepdims=True))
        p = O.bf16_round((p / p.sum(axis=1, keepdims=True)).astype(np.float32))
        top = -np.sort(-p, axis=1)[:, :10]
        top = O.bf16_round((top / top.sum(axis=1, keepdims=True)).astype(np.float32))
        rows.extend(top.astype(np.float64))
    edge = [
        [0.1] * 10,
        [0.5, 0.5] + [0.0] * 8,
        [1.0] + [0.0] * 9,
        [0.5, 0.25, 0.125, 0.0625, 0.03125, 0.015625, 0.0078125, 0.00390625, 0.001953125, 0.001953125],
        [0.25] * 4 + [0.0] * 6,
        [0.3, 0.3, 0.2, 0.1, 0.05, 0.05, 0.0, 0.0, 0.0, 0.0],
        [0.375, 0.25, 0.125, 0.125, 0.0625, 0.0625, 0.0, 0.0, 0.0, 0.0],
        [0.19921875, 0.19921875, 0.19921875, 0.10009765625, 0.10009765625, 0.0498046875,
         0.0498046875, 0.0498046875, 0.02490234375, 0.02490234375],
    ]
    rows.extend(np.asarray(edge, dtype=np.float64))
    return np.asarray(rows, dtype=np.float64)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    args = ap.parse_args()
    rows = weight_rows()
    sys.path.insert(0, os.path.abspath(args.reference))
    mlx = types.ModuleType("mlx")
    mlx.core = types.ModuleType("mlx.core")
    sys.modules["mlx"], sys.modules["mlx.core"] = mlx, mlx.core
    for name in ("compiled", "hostwindow"):
        sys.modules[f"models.flashnext.{name}"] = types.ModuleType(name)
    cache = types.ModuleType("expert_cache")
    cache._TIMERS = {}
    sys.modules["models.flashnext.expert_cache"] = cache
    from models.flashnext import adaptive_topk

    keeps = np.array([[adaptive_topk._keep_for_mass(r.tolist(), t) for r in rows] for t in THRESHOLDS],
                     dtype=np.int32)
    np.savez_compressed(os.path.join(HERE, "adaptive_keep.npz"), weights=rows,
                        thresholds=np.asarray(THRESHOLDS, dtype=np.float64), keeps=keeps)
    print(f"wrote {rows.shape[0]} rows x {len(THRESHOLDS)} thresholds; "
          f"keep counts {np.bincount(keeps.ravel()).tolist()}")


if __name__ == "__main__":
    main()
