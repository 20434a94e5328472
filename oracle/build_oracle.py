"""Build the C/OpenMP restatement (TEST INFRASTRUCTURE / CPU BASELINE ONLY).

    python oracle/build_oracle.py   ->  oracle/libvxcref.so
"""
from __future__ import annotations

import os
import shutil
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "vxmoe_cref.c")
LIB = os.path.join(HERE, "libvxcref.so")


def build(force: bool = False) -> str:
    if not force and os.path.exists(LIB) and os.path.getmtime(LIB) >= os.path.getmtime(SRC):
        return LIB
    cc = shutil.which("gcc") or "cc"
    cmd = [cc, "-O3", "-fopenmp", "-fPIC", "-shared", "-march=x86-64-v3", SRC, "-o", LIB, "-lm"]
    subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    print(build(force=True))
