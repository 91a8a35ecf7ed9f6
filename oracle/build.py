"""Build the C oracle (test infrastructure only): gcc -> oracle/_build/liboracle.so.

IEEE-strict flags (-ffp-contract=off -fno-fast-math) so every fmaf/add/div in oracle.c is
the single IEEE operation it spells. The reference itself is Python (nothing of it needs
compiling), so there is no ``oracle/_ref`` build for this path.
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "c", "oracle.c")
OUT_DIR = os.path.join(HERE, "_build")
LIB = os.path.join(OUT_DIR, "liboracle.so")


def build(force: bool = False) -> str:
    os.makedirs(OUT_DIR, exist_ok=True)
    if not force and os.path.exists(LIB) and os.path.getmtime(LIB) >= os.path.getmtime(SRC):
        return LIB
    cmd = ["gcc", "-O2", "-std=c11", "-fPIC", "-shared", "-ffp-contract=off", "-fno-fast-math",
           "-fno-builtin", "-o", LIB + ".tmp", SRC, "-lm"]
    subprocess.run(cmd, check=True)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
