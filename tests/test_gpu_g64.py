"""Native G64 records on the GPU (banks quantised in groups of 64 kept as
stored: one scale/bias pair per row and 64 inputs, 1152 record bytes per 16
rows x 128 inputs instead of 1280).

The pack kernel writes the oracle's G64 layout byte for byte.  A block over
native records returns the bits of the same layer expanded to groups of 32
(each pair repeated for both 32-input halves): the kernels sum per 32 inputs
in both forms and read the same scale for both halves, so the grouped GEMV,
the tcgen05 GEMM, the executor entry points and a slot pool all give
identical outputs and routing.  Against the G64 oracle the block meets the
block bar; a G64 checkpoint layer loads natively."""
from __future__ import annotations

import numpy as np
import pytest
import torch

import vxmoe_oracle as O
from helpers import assert_block_bar, bank_t, bf16_t, np32

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.fail("GPU tests need a CUDA device")
    import vxmoe
    vxmoe._lib.load()


def _bits(t):
    return t.view(torch.int16).cpu().numpy()


def _same(a, b, what):
    np.testing.assert_array_equal(_bits(a), _bits(b), err_msg=what)


def _weights(p, native, shared=True, device="cuda"):
    """MoEWeights of a G64 parameter set: native G64 banks, or every bank
    expanded to groups of 32 and packed; the shared-expert gate is expanded
    in both (the router side reads it in groups of 32)."""
    import vxmoe
    from vxmoe.ops import Q4Projection

    def proj(b, nat=native):
        return Q4Projection.from_group(*bank_t(b, device), p.group_size, native=nat)

    kw = {}
    if shared:
        kw = dict(shared_gate=proj(p.shared_gate), shared_up=proj(p.shared_up),
                  shared_down=proj(p.shared_down), shared_expert_gate=proj(p.shared_expert_gate, False))
    w = vxmoe.MoEWeights(proj(p.gate), proj(p.up), proj(p.down), router_w=bf16_t(p.router_w, device),
                         top_k=p.top_k, device=device, **kw)
    return w if native else w.pack()


@pytest.mark.parametrize("E,out,inn,tr,pair", [
    (3, 40, 128, 16, True), (2, 70, 192, 32, False), (2, 24, 64, 16, False),
    (4, 512, 2048, 16, True), (4, 2048, 512, 32, False)])
def test_pack_kernel_writes_the_oracle_g64_layout(E, out, inn, tr, pair):
    from vxmoe.ops import Q4Projection, tile_bank
    rng = np.random.default_rng(E + out + inn + 64)
    a = O.make_q4_bank(rng, E, out, inn, 64)
    b = O.make_q4_bank(rng, E, out, inn, 64) if pair else None
    rec = tile_bank(Q4Projection(*bank_t(a), 64), Q4Projection(*bank_t(b), 64) if pair else None, tr)
    torch.cuda.synchronize()
    assert rec.numel() == E * -(-out // tr) * -(-inn // 128) * (2 if pair else 1) * (tr // 16) * 1152
    np.testing.assert_array_equal(rec.cpu().numpy(), O.tile_records(a, b, tr, 64))


CFGS = [
    dict(seed=71, experts=32, hidden=256, inter=128, shared_inter=64, top_k=4, group_size=64),
    dict(seed=72, experts=16, hidden=192, inter=192, shared_inter=128, top_k=3, group_size=64),  # ragged chunks
]


@pytest.mark.parametrize("cfg", CFGS)
@pytest.mark.parametrize("down_rows", [32, 16])
def test_native_block_equals_expanded_block(cfg, down_rows):
    import vxmoe
    from vxmoe import _lib
    p = O.make_params(**cfg)
    nat, exp = _weights(p, True).pack(down_rows), _weights(p, False).pack(down_rows)
    assert nat.group_size == 64 and nat.pool.group_size == 64 and exp.group_size == 32
    assert nat.pool.nbytes() < exp.pool.nbytes()
    for path, Ts in ((_lib.PATH_GEMV, (1, 2, 7, 40)), (_lib.PATH_GEMM, (5, 64, 200))):
        for w in (nat, exp):
            w.expert_path = path
        for T in Ts:
            x = bf16_t(O.make_x(80 + T, T, p.hidden))
            y0, i0, w0 = vxmoe.moe_block(x, exp, return_routing=True)
            y1, i1, w1 = vxmoe.moe_block(x, nat, return_routing=True)
            torch.cuda.synchronize()
            np.testing.assert_array_equal(i0.cpu().numpy(), i1.cpu().numpy())
            _same(w1, w0, f"routing weights path {path} T={T}")
            _same(y1, y0, f"block path {path} T={T}")


def test_native_block_auto_path_meets_the_oracle_bar():
    """Under the automatic path: decode-sized batches take the multi-kernel
    GEMV (the single-launch decode kernel reads groups of 32 only), checked
    against the oracle's qmv arithmetic; from four routed positions per
    expert the tcgen05 GEMM, checked against its batched-matmul arithmetic."""
    import vxmoe
    p = O.make_params(**CFGS[0])
    w = _weights(p, True)
    for T in (1, 4, 33, 256):
        x = O.make_x(90 + T, T, p.hidden)
        y, inds, _ = vxmoe.moe_block(bf16_t(x), w, return_routing=True)
        logits = np32(vxmoe.router(bf16_t(x), w).logits)
        path = "prefill" if T * p.top_k >= 4 * p.num_experts else "decode"
        out = O.moe_block(x, p, logits=logits, path=path)
        np.testing.assert_array_equal(inds.cpu().numpy(), out.router.inds)
        ref64 = O.moe_block_reference_f64(x, p, out.router.inds, out.router.logits)
        scale = O.summand_scale(out.yd, out.router.weights, out.shared_y)
        assert_block_bar(np32(y), out.y, ref64, scale, f"native G64 {path} T={T}")


def test_native_executor_paths_equal_expanded():
    import vxmoe
    p = O.make_params(**dict(CFGS[0], seed=73))
    nat, exp = _weights(p, True, shared=False), _weights(p, False, shared=False)
    T = 9
    x = bf16_t(O.make_x(5, T, p.hidden))
    rng = np.random.default_rng(3)
    routes = torch.from_numpy(rng.integers(0, p.num_experts, (T, p.top_k)).astype(np.int32)).cuda()
    scores = bf16_t(O.bf16_round(rng.random((T, p.top_k)).astype(np.float32)))
    for kw in (dict(), dict(scores=scores)):
        _same(vxmoe.moe_experts(x, routes, nat, **kw), vxmoe.moe_experts(x, routes, exp, **kw),
              f"moe_experts {sorted(kw)}")
    half = torch.where(routes < 16, routes, torch.full_like(routes, -1))
    a = vxmoe.moe_experts_partial(x, half, scores, nat)
    b = vxmoe.moe_experts_partial(x, half, scores, exp)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(a.float().cpu().numpy(), b.float().cpu().numpy())


def test_native_slot_pool_layer_equals_resident_layer():
    import vxmoe
    p = O.make_params(**dict(CFGS[0], seed=74))
    full = _weights(p, True)
    part = _weights(p, True)
    pool = vxmoe.SlotPool(12, p.hidden, p.gate.w.shape[1], group_size=64)
    pool.attach(part)
    for T in (1, 3, 2):   # at most 12 distinct experts a call
        x = bf16_t(O.make_x(100 + T, T, p.hidden))
        _same(vxmoe.moe_block(x, part), vxmoe.moe_block(x, full), f"slot pool T={T}")
    assert pool.assigner.misses > 0
    with pytest.raises(ValueError):   # groups of 32 do not fit a G64 slot pool
        pool.attach(_weights(p, False))


def test_native_bank_without_pool_is_packed_and_bad_mixes_are_refused():
    import vxmoe
    from vxmoe.ops import Q4Projection
    p = O.make_params(**CFGS[0])
    w = _weights(p, True, shared=False)
    assert w.pool is not None and w.pool.group_size == 64
    g32 = Q4Projection.from_group(*bank_t(p.down), 64)
    with pytest.raises(ValueError):   # routed banks in two groupings
        vxmoe.MoEWeights(Q4Projection.from_group(*bank_t(p.gate), 64, native=True),
                         Q4Projection.from_group(*bank_t(p.up), 64, native=True), g32,
                         router_w=bf16_t(p.router_w), top_k=p.top_k)
