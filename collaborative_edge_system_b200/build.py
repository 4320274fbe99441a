"""Build libcea.so (the sm_100a kernels + C ABI) in place with nvcc.

    python -m collaborative_edge_system_b200.build [--force]

The library is written next to this file, so it travels with the source tree
to a GPU box; the build runs without a GPU (nvcc cross-compiles for sm_100a).
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libcea.so")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC,-O2", "-shared"]


def nvcc() -> str:
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(path):
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build libcea.so")
    return path


def sources():
    return [os.path.join(CSRC, f) for f in sorted(os.listdir(CSRC)) if f.endswith((".cu", ".cuh"))] + [
        os.path.join(INCLUDE, "cea.h")
    ]


def up_to_date() -> bool:
    if not os.path.exists(LIB):
        return False
    built = os.path.getmtime(LIB)
    return all(os.path.getmtime(s) <= built for s in sources())


def build(force: bool = False, verbose: bool = False, extra=()) -> str:
    if not force and up_to_date():
        return LIB
    tmp = LIB + ".tmp"
    cmd = [nvcc(), *ARCH, *FLAGS, *extra, "-I", INCLUDE, "-o", tmp, os.path.join(CSRC, "cea_api.cu"), "-lcudart", "-ldl"]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    if verbose and (res.stdout or res.stderr):
        print(res.stdout, res.stderr, flush=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    args = sys.argv[1:]
    extra = []
    if "--ptxas-v" in args:
        extra = ["-Xptxas", "-v"]
    print(build(force="--force" in args or bool(extra), verbose=True, extra=extra))
