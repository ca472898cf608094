"""Builds the sm_100a shared library libmoe_b200.so in-tree with nvcc.

Every kernel is compiled for sm_100a only (tcgen05 / TMA code has no other
target).  The library exports the C ABI declared in include/moe_ops.h.
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libmoe_b200.so")

SOURCES = ["routing.cu", "permute.cu", "grouped_gemm.cu", "combine.cu", "moe_ops.cu", "no_alloc.cu", "ep.cu"]
HEADERS = ["moe_common.cuh", "moe_kernels.h"]

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr"]
if os.environ.get("MOE_PTXAS_VERBOSE"):  # registers / spills / shared memory per kernel
    FLAGS = FLAGS + ["-Xptxas", "-v"]
# extra compile definitions, e.g. MOE_NVCC_EXTRA="-DMOE_GEMM_STAGES=3" (tuning builds)
FLAGS = FLAGS + os.environ.get("MOE_NVCC_EXTRA", "").split()


STAMP = os.path.join(BUILD, "flags.txt")


def _flags_changed() -> bool:
    """True when the objects were built with other flags (e.g. a tuning build)."""
    want = " ".join([NVCC, *ARCH, *FLAGS])
    have = open(STAMP).read() if os.path.exists(STAMP) else None
    return have != want


def _stale(out: str, deps: list[str]) -> bool:
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.getmtime(d) > t for d in deps)


def build(verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    include = os.path.join(os.path.dirname(HERE), "include")
    hdrs = [os.path.join(CSRC, h) for h in HEADERS] + [os.path.join(include, "moe_ops.h")]
    force = _flags_changed()
    objs = []
    for src in SOURCES:
        s = os.path.join(CSRC, src)
        o = os.path.join(BUILD, src.replace(".cu", ".o"))
        objs.append(o)
        if force or _stale(o, [s] + hdrs):
            cmd = [NVCC, *ARCH, *FLAGS, "-I", include, "-c", s, "-o", o]
            if verbose:
                print(" ".join(cmd), flush=True)
            subprocess.check_call(cmd)
    with open(STAMP, "w") as f:
        f.write(" ".join([NVCC, *ARCH, *FLAGS]))
    if force or _stale(LIB, objs):
        cmd = [NVCC, *ARCH, "-shared", "-cudart", "shared", "-o", LIB, *objs, "-lnccl"]
        if verbose:
            print(" ".join(cmd), flush=True)
        subprocess.check_call(cmd)
    return LIB


if __name__ == "__main__":
    print(build(verbose=True))
    sys.exit(0)
