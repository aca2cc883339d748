"""Builds libtrmoe.so in-tree (trochilus_b200/libtrmoe.so) with nvcc for sm_100a.

    python -m trochilus_b200.build          (or __graft_entry__.build())

One translation unit (csrc/capi.cu includes the kernel headers). -fmad=false: no floating-point
multiply-add is ever contracted, which the bit-exact paths rely on (they also spell every rounding
with an intrinsic). The CUDA runtime is linked statically, so the library needs only the driver.
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libtrmoe.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-fmad=false", "-prec-div=true", "-prec-sqrt=true", "-ftz=false",
         "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden", "-shared", "-cudart", "static"]


def sources():
    return [os.path.join(CSRC, f) for f in sorted(os.listdir(CSRC)) if f.endswith((".cu", ".cuh", ".h", ".inc"))]


def up_to_date() -> bool:
    if not os.path.exists(LIB):
        return False
    t = os.path.getmtime(LIB)
    return all(os.path.getmtime(s) <= t for s in sources() + [os.path.join(HERE, "..", "include", "trmoe.h"), __file__])


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and up_to_date():
        return LIB
    cmd = [NVCC, *ARCH, *FLAGS, "-I", os.path.join(HERE, "..", "include"), os.path.join(CSRC, "capi.cu"),
           "-o", LIB + ".tmp"]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), file=sys.stderr)
    subprocess.check_call(cmd)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
