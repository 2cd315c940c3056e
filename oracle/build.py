"""Compiles the C oracle (plstm_oracle.c) into oracle/lib/liboracle.so.

Test infrastructure only.  Built with gcc, OpenMP and a portable x86-64-v3
target (AVX2 + FMA) so that the library built here also runs on the GPU box's
host CPU.
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
SRC = os.path.join(HERE, "plstm_oracle.c")
LIB_DIR = os.path.join(HERE, "lib")
LIB = os.path.join(LIB_DIR, "liboracle.so")


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(LIB_DIR, exist_ok=True)
    if not force and os.path.exists(LIB) and os.path.getmtime(LIB) >= os.path.getmtime(SRC):
        return LIB
    cmd = ["gcc", "-O3", "-march=x86-64-v3", "-fopenmp", "-fPIC", "-shared", "-std=c11",
           "-o", LIB + ".tmp", SRC, "-lm"]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
