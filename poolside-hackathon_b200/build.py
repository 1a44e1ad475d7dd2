"""Build libkivi_sm100.so in-tree (nvcc, sm_100a only).

    python poolside-hackathon_b200/build.py [--force]

The library is plain C-ABI (include/kivi_sm100.h); it links the CUDA runtime
statically and resolves cuTensorMapEncodeTiled through the runtime's driver
entry-point query, so it has no dependency on torch or libcuda at link time.
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
LIB = os.path.join(HERE, "libkivi_sm100.so")
SOURCES = ["kivi_abi.cu", "kivi_quant.cu", "kivi_decode.cu", "kivi_paged.cu", "kivi_peer.cu"]
HEADERS = ["kivi_common.cuh", "kivi_internal.h"]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17",
         "-Xcompiler", "-fPIC", "-cudart", "static", "--expt-relaxed-constexpr"]


def _stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = [os.path.join(HERE, "csrc", f) for f in SOURCES + HEADERS]
    deps.append(os.path.join(ROOT, "include", "kivi_sm100.h"))
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and not _stale():
        return LIB
    objdir = os.path.join(HERE, "_build")
    os.makedirs(objdir, exist_ok=True)
    objs = []
    for s in SOURCES:
        o = os.path.join(objdir, s.replace(".cu", ".o"))
        cmd = [NVCC, *FLAGS, "-c", os.path.join(HERE, "csrc", s), "-o", o]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.check_call(cmd)
        objs.append(o)
    tmp = LIB + ".tmp"
    subprocess.check_call([NVCC, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-cudart", "static",
                           "-o", tmp, *objs])
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
