"""vx_moe_block_noalloc: the block for callers that cannot allocate device
memory (for example a plugin that runs inside another runtime's memory pool
and may not call cudaMalloc).  It must give the same result as vx_moe_block
with a caller workspace, call after call, while the static scratch array it
uses keeps whatever the previous call left in it.

This file is collected last on purpose, so a failure here comes after every
other test has run.  It builds its own inputs and also passes when run alone.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _call_noalloc(lib, x, w_struct, T, d, k, dev):
    y = torch.empty((T, d), dtype=torch.bfloat16, device=dev)
    inds = torch.empty((T, k), dtype=torch.int32, device=dev)
    wts = torch.empty((T, k), dtype=torch.bfloat16, device=dev)
    stream = torch.cuda.current_stream(dev).cuda_stream
    status = lib.vx_moe_block_noalloc(x.data_ptr(), T, ctypes.byref(w_struct), y.data_ptr(),
                                      inds.data_ptr(), wts.data_ptr(), stream)
    return status, y, inds, wts


@pytest.mark.parametrize("experts,hidden,inter,T", [(32, 256, 64, 5), (512, 2048, 512, 8)])
def test_noalloc_block_matches_workspace_block(experts, hidden, inter, T):
    if not torch.cuda.is_available():
        pytest.fail("this test needs a CUDA device")
    import vxmoe
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev)
    g.manual_seed(experts + T)
    w = vxmoe.MoEWeights.random(experts, hidden, inter, inter, 10 if experts >= 10 else 4,
                                device=dev, generator=g)
    lib = vxmoe._lib.load()
    st = w.vx()
    k = w.top_k
    for call in range(2):           # two calls in a row share the static scratch
        x = (torch.randn((T, hidden), device=dev, generator=g) * (1.0 + call)).to(torch.bfloat16)
        status, y, inds, wts = _call_noalloc(lib, x, st, T, hidden, k, dev)
        assert status == 0, lib.vx_strerror(status)
        y_ref, inds_ref, wts_ref = vxmoe.moe_block(x, w, return_routing=True)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(inds.cpu().numpy(), inds_ref.cpu().numpy())
        np.testing.assert_array_equal(wts.view(torch.int16).cpu().numpy(),
                                      wts_ref.view(torch.int16).cpu().numpy())
        # same kernels on the same inputs: identical bits (the repository's
        # block tolerance, normwise 1e-2, is far looser)
        np.testing.assert_array_equal(y.view(torch.int16).cpu().numpy(),
                                      y_ref.view(torch.int16).cpu().numpy())


def test_noalloc_block_rejects_a_batch_beyond_its_scratch():
    if not torch.cuda.is_available():
        pytest.fail("this test needs a CUDA device")
    import vxmoe
    dev = torch.device("cuda", 0)
    w = vxmoe.MoEWeights.random(64, 2048, 512, 512, 10, device=dev)
    lib = vxmoe._lib.load()
    st = w.vx()
    T = 4096   # far more scratch than VX_NOALLOC_SCRATCH_BYTES holds
    assert lib.vx_moe_block_workspace(T, ctypes.byref(st)) > (2 << 20)
    x = torch.zeros((T, 2048), dtype=torch.bfloat16, device=dev)
    status, _, _, _ = _call_noalloc(lib, x, st, T, 2048, 10, dev)
    assert status == vxmoe._lib.VX_EWORKSPACE
