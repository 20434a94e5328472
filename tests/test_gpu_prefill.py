"""Layer-major windows give the chunk-major result bit for bit: the grouped
GEMM computes each token's product with an expert independently of the other
tokens in its batch (the exactness argument of models/flashnext/
layer_major.py:16-22), so a window of chunks per layer equals chunk by chunk."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import vxmoe_oracle as O
from helpers import bf16_t, weights_from_oracle

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("packed", [True, False])
def test_layer_major_equals_chunk_major(packed):
    import vxmoe
    from vxmoe import prefill as P
    layers = []
    for i in range(3):
        p = O.make_params(seed=70 + i, experts=16, hidden=256, inter=128, shared_inter=64, top_k=4)
        w = weights_from_oracle(p)
        if packed:
            w.pack()
        gain = torch.ones(p.hidden, dtype=torch.bfloat16, device="cuda")
        layers.append(lambda h, w=w, gain=gain: h + vxmoe.moe_block(vxmoe.rms_norm(h, gain), w))
    x = bf16_t(O.make_x(73, 1500, 256))
    spans = P.plan_chunks(1500, 256)           # every chunk >= 64 tokens: the GEMM path (T*k >= 4E)
    a = P.run_chunk_major(layers, x, spans)
    b = P.run_layer_major(layers, x, spans, window=1024)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(a.view(torch.int16).cpu().numpy(), b.view(torch.int16).cpu().numpy())
