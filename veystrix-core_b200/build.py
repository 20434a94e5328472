"""Build libvxmoe.so for sm_100a, in-tree (vxmoe/lib/libvxmoe.so).

    python veystrix-core_b200/build.py [--force] [--verbose]

The library is a plain nvcc shared object with a C ABI (include/vxmoe.h);
the Python package loads it with ctypes.  Rebuilds only when a source is
newer than the library.
"""
from __future__ import annotations

import argparse
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(ROOT, "include")
LIBDIR = os.path.join(HERE, "vxmoe", "lib")
LIB = os.path.join(LIBDIR, "libvxmoe.so")

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-shared",
              "--expt-relaxed-constexpr", "-Xptxas", "-v"]


def sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def headers():
    return sorted(glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h"))
                  + glob.glob(os.path.join(INCLUDE, "*.h")))


def nvcc_path():
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def up_to_date():
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    return all(os.path.getmtime(p) <= t for p in sources() + headers() + [__file__])


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile every source to an object in parallel (one nvcc per file; no
    device code crosses files), then link the shared library."""
    if not force and up_to_date():
        return LIB
    os.makedirs(LIBDIR, exist_ok=True)
    import concurrent.futures
    import tempfile
    nvcc = nvcc_path()
    compile_flags = [f for f in NVCC_FLAGS if f != "-shared"]
    logs = []
    with tempfile.TemporaryDirectory(prefix="vxmoe_build_") as objdir:
        def compile_one(src):
            obj = os.path.join(objdir, os.path.basename(src) + ".o")
            cmd = [nvcc, *ARCH_FLAGS, *compile_flags, "-I", INCLUDE, "-I", CSRC, "-c", src, "-o", obj]
            proc = subprocess.run(cmd, capture_output=True, text=True)
            return src, obj, cmd, proc
        workers = max(1, min(len(sources()), os.cpu_count() or 1))
        with concurrent.futures.ThreadPoolExecutor(workers) as pool:
            results = list(pool.map(compile_one, sources()))
        failed = False
        for src, obj, cmd, proc in results:
            logs.append(" ".join(cmd) + "\n" + proc.stdout + proc.stderr)
            failed |= proc.returncode != 0
        tmp = LIB + ".tmp"
        if not failed:
            cmd = [nvcc, *ARCH_FLAGS, "-shared", "-Xcompiler", "-fPIC", *[r[1] for r in results],
                   "-o", tmp]
            proc = subprocess.run(cmd, capture_output=True, text=True)
            logs.append(" ".join(cmd) + "\n" + proc.stdout + proc.stderr)
            failed = proc.returncode != 0
    log = "\n".join(logs)
    with open(os.path.join(LIBDIR, "build.log"), "w") as fh:
        fh.write(log)
    if failed:
        sys.stderr.write(log)
        raise RuntimeError("nvcc failed building libvxmoe.so")
    if verbose:
        sys.stdout.write(log)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build(a.force, a.verbose))
