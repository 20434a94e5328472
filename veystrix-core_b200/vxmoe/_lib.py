"""ctypes binding of libvxmoe.so (the C ABI in include/vxmoe.h).

There is no fallback: if the library or a CUDA device is missing, every
compute call raises.  Loading the library itself needs no GPU.
"""
from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "lib", "libvxmoe.so")

VX_OK = 0
VX_EINVAL_SHAPE = 1
VX_EINVAL_DTYPE = 2
VX_EINVAL_INDEX = 3
VX_ECUDA = 4
VX_ETIMEOUT = 5
VX_EWORKSPACE = 6
VX_EUNSUPPORTED = 7

VX_DTYPE_BF16 = 0
VX_DTYPE_F32 = 1

c_int32 = ctypes.c_int32
c_int64 = ctypes.c_int64
c_size_t = ctypes.c_size_t
c_void_p = ctypes.c_void_p
c_float = ctypes.c_float


class VxQ4(ctypes.Structure):
    _fields_ = [
        ("w", c_void_p), ("scales", c_void_p), ("biases", c_void_p),
        ("experts", c_int32), ("out", c_int32), ("in_", c_int32), ("group_size", c_int32),
    ]


class VxQ4Tiles(ctypes.Structure):
    _fields_ = [
        ("records", c_void_p), ("experts", c_int32), ("out", c_int32), ("in_", c_int32),
        ("group_size", c_int32), ("nproj", c_int32), ("tile_rows", c_int32),
    ]


class VxMoEPool(ctypes.Structure):
    _fields_ = [
        ("gate_up", VxQ4Tiles), ("down", VxQ4Tiles),
        ("shared_gate_up", VxQ4Tiles), ("shared_down", VxQ4Tiles),
        ("slot_of", c_void_p), ("slots", c_int32),
    ]


class VxMoEWeights(ctypes.Structure):
    _fields_ = [
        ("gate", VxQ4), ("up", VxQ4), ("down", VxQ4),
        ("shared_gate", VxQ4), ("shared_up", VxQ4), ("shared_down", VxQ4),
        ("shared_expert_gate", VxQ4),
        ("router_w", c_void_p),
        ("num_experts", c_int32), ("hidden", c_int32), ("top_k", c_int32),
        ("pool", ctypes.POINTER(VxMoEPool)),
        ("expert_path", c_int32),
        ("router_bias", c_void_p),
        ("keep_mass", ctypes.c_double),
        ("keep_min", c_int32),
    ]


PATH_AUTO, PATH_GEMV, PATH_GEMM = 0, 1, 2

EP_MAX_RANKS = 8
EP_IPC_HANDLE_BYTES = 64


class VxEpComm(ctypes.Structure):
    _fields_ = [
        ("buffers", c_void_p * EP_MAX_RANKS),
        ("rank", c_int32), ("world", c_int32), ("tokens_cap", c_int32),
        ("hidden", c_int32), ("top_k", c_int32), ("num_experts", c_int32),
        ("err", c_void_p), ("wait_ns", ctypes.c_uint64),
    ]


P = c_void_p
# name: (restype, argtypes)
SIGNATURES = {
    "vx_version": (ctypes.c_char_p, []),
    "vx_strerror": (ctypes.c_char_p, [ctypes.c_int]),
    "vx_last_cuda_error": (ctypes.c_char_p, []),
    "vx_q4_tiles_bytes": (c_size_t, [c_int32, c_int32, c_int32, c_int32, c_int32]),
    "vx_q4_tiles_bytes_group": (c_size_t, [c_int32, c_int32, c_int32, c_int32, c_int32, c_int32]),
    "vx_q4_tile": (ctypes.c_int, [ctypes.POINTER(VxQ4), ctypes.POINTER(VxQ4), c_int32, c_int32,
                                  P, c_size_t, P]),
    "vx_q4_dequant": (ctypes.c_int, [ctypes.POINTER(VxQ4), c_int32, P, P]),
    "vx_swiglu_bf16": (ctypes.c_int, [P, P, P, c_int64, P]),
    "vx_gather_qmm_workspace": (c_size_t, [c_int64, c_int32, c_int32, c_int64, c_int32]),
    "vx_gather_qmm": (ctypes.c_int, [P, c_int64, ctypes.POINTER(VxQ4), P, P, c_int64, c_int32,
                                     c_int32, P, P, c_size_t, P]),
    "vx_softmax_topk": (ctypes.c_int, [P, c_int32, c_int32, c_int32, P, P, P, P, P]),
    "vx_router_workspace": (c_size_t, [c_int32, ctypes.POINTER(VxMoEWeights)]),
    "vx_router": (ctypes.c_int, [P, c_int32, ctypes.POINTER(VxMoEWeights), P, P, P, P, P,
                                 c_size_t, P]),
    "vx_permute_workspace": (c_size_t, [c_int64, c_int32]),
    "vx_permute": (ctypes.c_int, [P, c_int64, c_int32, P, P, P, P, P, c_size_t, P]),
    "vx_moe_experts_workspace": (c_size_t, [c_int32, ctypes.POINTER(VxMoEWeights)]),
    "vx_moe_experts": (ctypes.c_int, [P, c_int32, P, P, ctypes.POINTER(VxMoEWeights), P, P, P,
                                      P, P, c_size_t, P]),
    "vx_moe_experts_partial": (ctypes.c_int, [P, c_int32, P, P, ctypes.POINTER(VxMoEWeights), P,
                                              P, c_size_t, P]),
    "vx_moe_block_workspace": (c_size_t, [c_int32, ctypes.POINTER(VxMoEWeights)]),
    "vx_moe_block": (ctypes.c_int, [P, c_int32, ctypes.POINTER(VxMoEWeights), P, P, P, P,
                                    c_size_t, P]),
    "vx_moe_block_noalloc": (ctypes.c_int, [P, c_int32, ctypes.POINTER(VxMoEWeights), P, P, P,
                                            P]),
    "vx_ep_buffer_bytes": (c_size_t, [c_int32, c_int32, c_int32, c_int32]),
    "vx_ep_ipc_handle": (ctypes.c_int, [P, P, ctypes.POINTER(ctypes.c_uint64)]),
    "vx_ep_ipc_open": (ctypes.c_int, [P, ctypes.c_uint64, ctypes.POINTER(c_void_p)]),
    "vx_ep_ipc_close": (ctypes.c_int, [P, ctypes.c_uint64]),
    "vx_ep_dispatch": (ctypes.c_int, [ctypes.POINTER(VxEpComm), P, c_int32, P, P, P]),
    "vx_ep_experts_workspace": (c_size_t, [ctypes.POINTER(VxEpComm), c_int32,
                                           ctypes.POINTER(VxMoEWeights)]),
    "vx_ep_experts": (ctypes.c_int, [ctypes.POINTER(VxEpComm), c_int32,
                                     ctypes.POINTER(VxMoEWeights), P, c_size_t, P]),
    "vx_ep_combine": (ctypes.c_int, [ctypes.POINTER(VxEpComm), c_int32, P, P, P, P, P]),
    "vx_rmsnorm": (ctypes.c_int, [P, P, c_int32, c_int32, c_float, P, P]),
    "vx_weighted_combine": (ctypes.c_int, [P, c_int32, c_int32, P, P, c_int64, c_int32, c_int32, P, P, P]),
    "vx_profile_enable": (ctypes.c_int, [ctypes.c_int]),
    "vx_profile_read": (ctypes.c_int, [ctypes.c_int, ctypes.c_char_p, ctypes.c_int,
                                       ctypes.POINTER(ctypes.c_double),
                                       ctypes.POINTER(c_int32), ctypes.POINTER(c_int32)]),
}

_lock = threading.Lock()
_lib = None


def load():
    """Load libvxmoe.so and bind every C ABI symbol."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"libvxmoe.so is not built ({LIB_PATH}); run veystrix-core_b200/build.py")
        lib = ctypes.CDLL(LIB_PATH)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def exported_symbols():
    return sorted(SIGNATURES)


def check(status: int, what: str = "") -> None:
    """Map a vx_status onto the exception the reference raises for it."""
    if status == VX_OK:
        return
    lib = load()
    msg = lib.vx_strerror(status).decode()
    if what:
        msg = f"{what}: {msg}"
    if status in (VX_EINVAL_SHAPE, VX_EINVAL_INDEX, VX_EWORKSPACE):
        raise ValueError(msg)
    if status == VX_EINVAL_DTYPE:
        raise TypeError(msg)
    if status == VX_ECUDA:
        msg += f" ({lib.vx_last_cuda_error().decode()})"
    raise RuntimeError(msg)


def profile_enable(enabled: bool = True) -> None:
    """Start (and reset) or stop per-stage CUDA-event timing."""
    check(load().vx_profile_enable(int(bool(enabled))), "profile_enable")


def profile_read(max_stages: int = 32) -> dict:
    """{stage label: (launches, average ms)} since the last enable."""
    lib = load()
    labels = ctypes.create_string_buffer(4096)
    avg = (ctypes.c_double * max_stages)()
    cnt = (c_int32 * max_stages)()
    n = c_int32(0)
    check(lib.vx_profile_read(max_stages, labels, 4096, avg, cnt, ctypes.byref(n)), "profile_read")
    names = labels.value.decode().split("\n")[: n.value]
    return {name: (int(cnt[i]), float(avg[i])) for i, name in enumerate(names)}
