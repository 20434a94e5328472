"""The build's smoke entry point on the GPU: one small block on cuda:0 in the
MLX layout and again from the tiled pool, checked against the CPU oracle
(top-k ids exact, outputs within the block bar) and against each other
(same routing; the same products, so most outputs keep their bits)."""
from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_smoke_entry_point():
    if not torch.cuda.is_available():
        pytest.fail("GPU tests need a CUDA device")
    import __graft_entry__
    __graft_entry__.smoke()
