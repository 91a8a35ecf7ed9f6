"""Build the C-ABI shared library libb200moe.so in-tree with nvcc for sm_100a.

One shared object from every ``csrc/*.cu``; static cudart; the public header is
``include/b200moe.h``. The library sits next to this file so it travels with the repo.
"""
from __future__ import annotations

import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libb200moe.so")
BUILD_DIR = os.path.join(HERE, "_build")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         "-I", os.path.join(ROOT, "include"), "-I", CSRC]


def sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _stale() -> bool:
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = sources() + glob.glob(os.path.join(CSRC, "*.cuh")) + [os.path.join(ROOT, "include", "b200moe.h")]
    return any(os.path.getmtime(p) > t for p in deps)


def build(force: bool = False, verbose: bool = False, ptxas_v: bool = False) -> str:
    if not force and not _stale():
        return LIB
    os.makedirs(BUILD_DIR, exist_ok=True)
    objs = []
    for src in sources():
        obj = os.path.join(BUILD_DIR, os.path.basename(src) + ".o")
        cmd = [NVCC, *ARCH, *FLAGS, "-c", src, "-o", obj]
        if ptxas_v:
            cmd += ["-Xptxas", "-v"]
        if verbose:
            print(" ".join(cmd))
        subprocess.run(cmd, check=True)
        objs.append(obj)
    tmp = LIB + ".tmp"
    subprocess.run([NVCC, *ARCH, "-shared", "-o", tmp, *objs], check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv, ptxas_v="--ptxas" in sys.argv))
