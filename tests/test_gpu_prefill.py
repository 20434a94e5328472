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


def test_budgeted_plan_with_the_block_memory_model():
    """The budgeted policy sized by the block's own scratch: every chunk's
    increment fits the budget, and the chunked run equals one call over the
    whole prompt bit for bit (every chunk takes the GEMM path)."""
    import vxmoe
    from vxmoe import prefill as P
    p = O.make_params(seed=80, experts=16, hidden=256, inter=128, shared_inter=64, top_k=4)
    w = weights_from_oracle(p)
    w.pack()
    model = P.block_memory_model(w, pair_bytes=3072)   # an attention term of a larger model
    budget = model.increment(1024, 1200)        # 2048 never fits; 1024 fits up to position 1200
    spans = P.plan_chunks(3000, 0, policy="budgeted", budget=budget, model=model)
    sizes = [e - s for s, e in spans]
    assert sizes == [1024, 1024, 512, 440]
    assert all(model.increment(e - s, s) <= budget for s, e in spans[:-1])
    assert model.increment(2048, 0) > budget and model.increment(1024, 2048) > budget
    x = bf16_t(O.make_x(81, 3000, 256))
    whole = vxmoe.moe_block(x, w)
    chunked = torch.cat([vxmoe.moe_block(x[s:e], w) for s, e in spans])
    assert torch.equal(whole, chunked)
