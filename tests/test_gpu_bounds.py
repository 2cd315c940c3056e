"""The bounds-check build of the library (lib/libplstm_bc.so, compiled with
-DPLSTM_BOUNDS_CHECK): the tensor-core wavefront kernel tests the index of every
global, shared and distributed-shared access it makes against its buffer's extent
and reports PLSTM_EBOUNDS (with the checking site) instead of faulting.  Small
shapes covering every tile plan (two 16-row slots, three 16-row slots, two 32-row
slots, the device-side height choice), output mode, variable lengths, initial
state, input widths (read by the x warp or repacked), hidden sizes and layer
counts run through it in a separate process (the library is loaded once per
process); every call synchronises and must report no violation and match the
oracle.  compute-sanitizer is not available on this pool; this is its stand-in for
the index arithmetic of these kernels."""
from __future__ import annotations

import os
import subprocess
import sys

import pytest

from conftest import ROOT

pytestmark = pytest.mark.gpu

SCRIPT = r"""
import os, sys
root, tests = sys.argv[1], sys.argv[2]
sys.path[:0] = [root, tests]
import numpy as np, torch
from persistent_lstm_hip_b200 import _lib, core
from helpers import make_model, weights_of, oracle_of, assert_close16
assert _lib.LIB_PATH.endswith("libplstm_bc.so"), _lib.LIB_PATH
dev = torch.device("cuda:0")
cases = [
    # B, T, I, H, L, mode, varlen, hx, dtype, forced tile rows
    (5, 9, 5, 128, 1, "last", False, False, torch.float16, None),
    (33, 12, 5, 128, 4, "seq", True, True, torch.float16, None),
    (100, 10, 20, 100, 2, "hseq", True, False, torch.bfloat16, None),
    (300, 8, 5, 128, 3, "seq", False, True, torch.float16, None),
    (520, 7, 5, 128, 4, "last", False, False, torch.float16, None),
    (700, 6, 5, 128, 4, "hseq", True, True, torch.float16, None),
    (520, 9, 5, 128, 4, "seq", True, False, torch.float16, None),
    (64, 8, 128, 64, 2, "seq", False, False, torch.float16, None),
    (40, 6, 5, 128, 6, "last", True, False, torch.float16, None),
    (96, 7, 5, 128, 2, "seq", True, True, torch.float16, 32),
    (96, 7, 5, 128, 2, "seq", True, True, torch.float16, 48),
    (96, 7, 5, 128, 2, "seq", True, True, torch.float16, 64),
    (24, 6, 5, 256, 2, "seq", True, True, torch.float16, None),
    (24, 5, 9, 512, 1, "last", False, False, torch.bfloat16, None),
]
for i, (B, T, I, H, L, mode, varlen, hx, dt, ntile) in enumerate(cases):
    if ntile:
        os.environ["PLSTM_TC_NTILE"] = str(ntile)
    else:
        os.environ.pop("PLSTM_TC_NTILE", None)
    w = weights_of(make_model(I, H, L, 24, seed=i), L, dt, dev)
    g = torch.Generator().manual_seed(100 + i)
    x = torch.randn(B, T, I, generator=g).to(dev, dt)
    lens = torch.randint(1, T + 1, (B,), generator=g, dtype=torch.int32) if varlen else None
    h = None
    if hx:
        h = ((0.5 * torch.randn(L, B, H, generator=g)).to(dev, dt), (0.5 * torch.randn(L, B, H, generator=g)).to(dev, dt))
    pw = core.PackedWeights(*w, out_mode=mode, backend="tc")
    out, h_n, c_n = pw.forward(x, lengths=None if lens is None else lens.to(dev), hx=h, check=True)
    r_out, r_h, r_c = oracle_of(x, *w, lengths=lens, hx=h, out_mode=mode)
    assert_close16(out, r_out, f"case {i} out")
    assert_close16(h_n, r_h, f"case {i} h_n")
    assert_close16(c_n, r_c, f"case {i} c_n")
print("bounds-check build: %d cases, no violation" % len(cases))
"""


def test_bounds_check_build_small_shapes(cuda_device):
    lib = os.path.join(ROOT, "persistent_lstm_hip_b200", "lib", "libplstm_bc.so")
    if not os.path.exists(lib):
        pytest.fail(f"{lib} is missing: build it with __graft_entry__.build()")
    env = dict(os.environ, PLSTM_LIB=lib)
    env.pop("PLSTM_TC_NTILE", None)
    r = subprocess.run([sys.executable, "-c", SCRIPT, ROOT, os.path.join(ROOT, "tests")], env=env,
                       capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, (r.stdout[-3000:] + r.stderr[-3000:])
    assert "no violation" in r.stdout
