"""The C/OpenMP restatement (CPU baseline) against the NumPy oracle."""
from __future__ import annotations

import numpy as np

import vxmoe_oracle as O


def test_c_restatement_matches_numpy_oracle():
    import vxmoe_cref as C
    for seed, (E, d, I, k, T) in enumerate([(32, 256, 64, 4, 5), (64, 512, 128, 10, 9)]):
        p = O.make_params(seed=seed, experts=E, hidden=d, inter=I, shared_inter=I, top_k=k)
        x = O.make_x(seed + 7, T, d)
        y = C.Block(p)(x)
        ref = O.moe_block(x, p)
        assert O.normwise_error(y, ref.y) < 1e-2
        assert C.threads() >= 1
