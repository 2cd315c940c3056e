"""Builds oracle/_ref/libplstm_ref.so: the reference's own CPU implementation of the
fixed 4-layer path (persistent_lstm_hip/csrc/persistent_lstm_reference.cpp, compiled
from the reference checkout where it lies) plus the C entry point of ref_shim.cpp.

Test and benchmark infrastructure only.  It needs the reference checkout, so it runs
where that checkout is mounted (the build container); the built library then travels
with the repository snapshot (oracle/_ref is git-ignored).  The reference file
includes <torch/extension.h>, so it is compiled against the installed torch's headers
and linked against its libtorch (the library the reference itself links); nothing of
the reference's own build system is run.
"""
from __future__ import annotations

import os
import subprocess
import sys
import sysconfig

HERE = os.path.dirname(os.path.abspath(__file__))
REF_CSRC = os.path.join(os.sep, "root", "reference", "persistent_lstm_hip", "csrc")
REF_SRC = os.path.join(REF_CSRC, "persistent_lstm_reference.cpp")
SHIM = os.path.join(HERE, "ref_shim.cpp")
OUT_DIR = os.path.join(HERE, "_ref")
LIB = os.path.join(OUT_DIR, "libplstm_ref.so")


def available() -> bool:
    return os.path.exists(REF_SRC)


def build(force: bool = False, verbose: bool = False) -> str:
    """Compiles the library if the reference source is present; returns its path."""
    if not available():
        raise FileNotFoundError(f"{REF_SRC} is not present (the reference checkout is mounted only where "
                                "the repository is built)")
    os.makedirs(OUT_DIR, exist_ok=True)
    newest = max(os.path.getmtime(REF_SRC), os.path.getmtime(SHIM))
    if not force and os.path.exists(LIB) and os.path.getmtime(LIB) >= newest:
        return LIB
    import torch
    from torch.utils import cpp_extension as ce

    incs = ce.include_paths() + [sysconfig.get_paths()["include"], REF_CSRC]
    libdir = ce.library_paths()[0]
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           "-DTORCH_EXTENSION_NAME=plstm_ref", *[f"-I{d}" for d in incs], "-o", LIB + ".tmp", REF_SRC, SHIM,
           f"-L{libdir}", f"-Wl,-rpath,{libdir}", "-ltorch", "-ltorch_cpu", "-lc10"]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    os.replace(LIB + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
