"""ctypes wrapper of the C/OpenMP restatement (TEST INFRASTRUCTURE / CPU
BASELINE ONLY): the block of ``vxmoe_oracle`` at native speed on the host
cores, used as ``bench.py``'s CPU baseline and checked against the NumPy
oracle in ``tests/``."""
from __future__ import annotations

import ctypes
import os

import numpy as np

import vxmoe_oracle as O

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "libvxcref.so")


class _Q4(ctypes.Structure):
    _fields_ = [("w", ctypes.c_void_p), ("s", ctypes.c_void_p), ("b", ctypes.c_void_p),
                ("experts", ctypes.c_int), ("out", ctypes.c_int), ("in_", ctypes.c_int)]


_lib = None


def _load():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB):
            from build_oracle import build
            build()
        lib = ctypes.CDLL(LIB)
        lib.vx_cref_block.restype = ctypes.c_int
        lib.vx_cref_block.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                      ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_void_p] + \
            [_Q4] * 7 + [ctypes.c_void_p]
        lib.vx_cref_threads.restype = ctypes.c_int
        _lib = lib
    return _lib


def threads() -> int:
    return int(_load().vx_cref_threads())


class Block:
    """Holds contiguous float32/uint32 copies of one layer's parameters."""

    def __init__(self, p: "O.MoEParams"):
        self.p = p
        self._keep = []
        self.banks = [self._q4(b) for b in (p.gate, p.up, p.down, p.shared_gate, p.shared_up,
                                            p.shared_down, p.shared_expert_gate)]
        self.router = np.ascontiguousarray(p.router_w, dtype=np.float32)

    def _q4(self, b: "O.Q4Bank") -> _Q4:
        w = np.ascontiguousarray(b.w, dtype=np.uint32)
        s = np.ascontiguousarray(b.scales, dtype=np.float32)
        bb = np.ascontiguousarray(b.biases, dtype=np.float32)
        self._keep += [w, s, bb]
        return _Q4(w.ctypes.data, s.ctypes.data, bb.ctypes.data, w.shape[0], w.shape[1], w.shape[2] * 8)

    def __call__(self, x) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        T, d = x.shape
        y = np.empty((T, d), np.float32)
        p = self.p
        rc = _load().vx_cref_block(x.ctypes.data, T, p.num_experts, d, p.gate.w.shape[1],
                                   p.shared_gate.w.shape[1], p.top_k, self.router.ctypes.data,
                                   *self.banks, y.ctypes.data)
        if rc:
            raise RuntimeError(f"vx_cref_block failed ({rc})")
        return y


def block_runner(seed: int = 0):
    return Block(O.make_params(seed=seed))
