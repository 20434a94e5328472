"""CPU-only checks of the C ABI library and the host layer (no GPU calls)."""
from __future__ import annotations

import ctypes
import os
import re
from types import SimpleNamespace

import numpy as np
import pytest

from conftest import ROOT

HEADER = os.path.join(ROOT, "include", "vxmoe.h")


def _header_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(vx_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    from vxmoe import _lib
    return _lib.load()


def test_library_exports_every_declared_symbol(lib):
    from vxmoe import _lib
    declared = _header_functions()
    assert declared, "no functions parsed from vxmoe.h"
    for name in declared:
        assert hasattr(lib, name), f"libvxmoe.so does not export {name}"
    assert sorted(declared) == sorted(_lib.exported_symbols())


def test_version_and_error_strings(lib):
    assert lib.vx_version().decode().startswith("vxmoe")
    assert lib.vx_strerror(0).decode() == "ok"
    assert "workspace" in lib.vx_strerror(6).decode()


def test_library_is_built_for_sm100a():
    from vxmoe import _lib
    log = open(os.path.join(os.path.dirname(_lib.LIB_PATH), "build.log")).read()
    assert "arch=compute_100a,code=sm_100a" in log


def test_workspace_sizes_are_consistent(lib):
    from vxmoe._lib import VxMoEWeights, VxQ4
    w = VxMoEWeights()
    w.num_experts, w.hidden, w.top_k = 512, 2048, 10
    w.gate = VxQ4(0, 0, 0, 512, 512, 2048, 32)
    w.up = VxQ4(0, 0, 0, 512, 512, 2048, 32)
    w.down = VxQ4(0, 0, 0, 512, 2048, 512, 32)
    small = lib.vx_moe_block_workspace(1, ctypes.byref(w))
    big = lib.vx_moe_block_workspace(64, ctypes.byref(w))
    assert 0 < small < big
    # h and yd dominate: (T*k) * (I + d) * 2 bytes
    assert big >= 64 * 10 * (512 + 2048) * 2
    assert lib.vx_gather_qmm_workspace(10, 1, 512, 10, 2048) > 10 * 2048 * 2
    assert lib.vx_permute_workspace(100, 512) > 0


def test_abi_rejects_bad_arguments_without_touching_the_device(lib):
    from vxmoe._lib import VX_EINVAL_SHAPE, VX_EWORKSPACE, VX_EUNSUPPORTED, VxQ4
    # k > E
    assert lib.vx_softmax_topk(None, 4, 8, 9, None, None, None, None, None) == VX_EINVAL_SHAPE
    # E too large
    assert lib.vx_softmax_topk(None, 4, 4096, 2, None, None, None, None, None) == VX_EINVAL_SHAPE
    # null weights
    assert lib.vx_moe_block(None, 1, None, None, None, None, None, 0, None) == VX_EINVAL_SHAPE
    # group size 64 is not supported by the kernels
    q = VxQ4(16, 16, 16, 2, 4, 64, 64)
    assert lib.vx_gather_qmm(None, 0, ctypes.byref(q), None, None, 1, 1, 0, None, None, 0,
                             None) == VX_EUNSUPPORTED
    # empty batch is a no-op
    q = VxQ4(16, 16, 16, 2, 4, 64, 32)
    assert lib.vx_gather_qmm(None, 0, ctypes.byref(q), None, None, 0, 1, 0, None, None, 0, None) == 0
    # workspace too small
    assert lib.vx_permute(None, 0, 4, None, None, ctypes.c_void_p(16), None, None, 0,
                          None) == VX_EWORKSPACE


def test_status_maps_onto_reference_exceptions():
    from vxmoe import _lib
    _lib.check(0)
    with pytest.raises(ValueError):
        _lib.check(_lib.VX_EINVAL_SHAPE)
    with pytest.raises(TypeError):
        _lib.check(_lib.VX_EINVAL_DTYPE)
    with pytest.raises(RuntimeError):
        _lib.check(_lib.VX_EUNSUPPORTED)


def test_executor_constructor_bounds():
    from vxmoe import MoEExecutor
    for kwargs in ({"expert_count": 0, "hidden_size": 2, "top_k": 1},
                   {"expert_count": 2, "hidden_size": 0, "top_k": 1},
                   {"expert_count": 2, "hidden_size": 2, "top_k": 0}):
        with pytest.raises(ValueError):
            MoEExecutor(**kwargs)
    with pytest.raises(ValueError):
        MoEExecutor(expert_count=2, hidden_size=2, top_k=3)
    with pytest.raises(ValueError):
        MoEExecutor(expert_count=2, hidden_size=32, top_k=1, group_size=48)


def test_executor_capabilities_and_unavailable_backend():
    from vxmoe import MoEExecutor, probe_capabilities
    caps = probe_capabilities(SimpleNamespace(available=False, supports_custom_moe=False))
    assert not caps.available and not caps.supports_custom_moe
    ex = MoEExecutor(2, 2, 1, backend=SimpleNamespace(available=True, supports_custom_moe=False))
    with pytest.raises(RuntimeError, match="custom MoE"):
        ex.execute(np.zeros((1, 2), np.float32), np.zeros((1, 1), np.int32),
                   np.ones((1, 1), np.float32))


def test_executor_validation_errors_before_device_work():
    from vxmoe import MoEExecutor
    ex = MoEExecutor(expert_count=2, hidden_size=32, top_k=1,
                     backend=SimpleNamespace(available=True, supports_custom_moe=True))
    with pytest.raises(ValueError, match="same token count"):
        ex.execute(np.zeros((2, 32), np.float32), np.zeros((1, 1), np.int32), {})
    with pytest.raises(ValueError, match="shape"):
        ex.execute(np.zeros((1, 16), np.float32), np.zeros((1, 1), np.int32), {})
    with pytest.raises(ValueError, match="together"):
        ex.execute(np.zeros((1, 32), np.float32), np.zeros((1, 1), np.int32), {},
                   shared=np.zeros((1, 32)))
    with pytest.raises(TypeError):
        ex.execute(np.zeros((1, 32), np.float32), np.zeros((1, 1), np.int32))


def test_executor_combine_only_form_matches_reference_values(golden_dir):
    from vxmoe import MoEExecutor
    g = np.load(os.path.join(golden_dir, "combine.npz"))
    ex = MoEExecutor(3, 2, 2, backend=SimpleNamespace(available=True, supports_custom_moe=True))
    out = ex.execute(g["eo"], g["r"], g["sc"])
    np.testing.assert_array_equal(out, np.array([[25.75, 51.5], [192.0, 256.0]], np.float32))
    assert ex.last_path == "custom-cuda"


def test_weighted_combine_numpy_matches_golden(golden_dir):
    from vxmoe import weighted_combine
    g = np.load(os.path.join(golden_dir, "combine.npz"))
    np.testing.assert_array_equal(weighted_combine(g["eo2"], g["r2"], g["sc2"]), g["c2"])
    np.testing.assert_array_equal(weighted_combine(g["slot"], g["r3"], g["sc3"]), g["c3"])
    with pytest.raises(ValueError):
        weighted_combine(np.zeros((2, 3, 2)), np.array([[0, 3]]), np.ones((1, 2)))


def test_build_executor_infers_dimensions_from_packs():
    from vxmoe import build_executor
    packs = {
        "gate_proj": (np.zeros((4, 8, 8), np.uint32), None, None),
        "up_proj": (np.zeros((4, 8, 8), np.uint32), None, None),
        "down_proj": (np.zeros((4, 64, 1), np.uint32), None, None),
    }
    ex = build_executor(packs=packs, group_size=32, bits=4, mode="affine", top_k=2,
                        backend=SimpleNamespace(available=True, supports_custom_moe=True))
    assert (ex.expert_count, ex.hidden_size, ex.top_k) == (4, 64, 2)
    with pytest.raises(ValueError):
        build_executor(packs=packs, bits=8)
