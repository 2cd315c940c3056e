"""Builds the in-tree CUDA library persistent_lstm_hip_b200/lib/libplstm.so.

Every translation unit is compiled for sm_100a only
(`-gencode arch=compute_100a,code=sm_100a`); nvcc cross-compiles without a
GPU.  The library has no torch dependency: it exports the C ABI of
include/plstm.h and is loaded with ctypes.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB_DIR = os.path.join(HERE, "lib")
OBJ_DIR = os.path.join(HERE, "lib", "obj")
LIB = os.path.join(LIB_DIR, "libplstm.so")
OBJ_DIR_BC = os.path.join(HERE, "lib", "obj_bc")
LIB_BC = os.path.join(LIB_DIR, "libplstm_bc.so")
SOURCES = ["plstm_abi.cu", "plstm_simt.cu", "plstm_tc.cu", "plstm_tcl.cu", "plstm_gemm.cu", "plstm_misc.cu",
           "plstm_noalloc.cu", "plstm_dedupe.cu"]
HEADERS = ["plstm_common.cuh", "sm100_ptx.cuh"]
NVCC = os.environ.get("NVCC", "nvcc")
FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-lineinfo", "-std=c++17",
         "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden", "--expt-relaxed-constexpr",
         "-I", os.path.join(ROOT, "include")]


def _stale(target: str, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src: str, verbose: bool, bounds_check: bool = False) -> str:
    obj_dir = OBJ_DIR_BC if bounds_check else OBJ_DIR
    obj = os.path.join(obj_dir, os.path.splitext(src)[0] + ".o")
    deps = [os.path.join(CSRC, src)] + [os.path.join(CSRC, h) for h in HEADERS] + \
        [os.path.join(ROOT, "include", "plstm.h")]
    if _stale(obj, deps):
        cmd = [NVCC, *FLAGS, *(["-DPLSTM_BOUNDS_CHECK"] if bounds_check else []), "-c", os.path.join(CSRC, src),
               "-o", obj]
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        subprocess.run(cmd, check=True)
    return obj


def build(force: bool = False, verbose: bool = False, bounds_check: bool = False) -> str:
    """Builds lib/libplstm.so, or with bounds_check=True lib/libplstm_bc.so: the same sources
    compiled with -DPLSTM_BOUNDS_CHECK, whose kernels test the indices of their global, shared
    and distributed-shared accesses and report PLSTM_EBOUNDS instead of faulting (the tests run
    small shapes through it)."""
    obj_dir, lib = (OBJ_DIR_BC, LIB_BC) if bounds_check else (OBJ_DIR, LIB)
    os.makedirs(obj_dir, exist_ok=True)
    if force:
        for f in os.listdir(obj_dir):
            os.remove(os.path.join(obj_dir, f))
    with cf.ThreadPoolExecutor(max_workers=len(SOURCES)) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose, bounds_check), SOURCES))
    if force or _stale(lib, objs):
        cmd = [NVCC, "-shared", "-gencode", "arch=compute_100a,code=sm_100a", "-o", lib + ".tmp", *objs,
               "-lcudart"]
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        subprocess.run(cmd, check=True)
        os.replace(lib + ".tmp", lib)
    return lib


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True, bounds_check="--bounds-check" in sys.argv))
