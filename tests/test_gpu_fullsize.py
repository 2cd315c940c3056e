"""Full-size parity: the BASELINE configurations at their own sizes (T = 1000 dependent
steps), against the f64 oracle (pinned to the reference's outputs in test_oracle.py).

Error growth over a thousand dependent steps in four layers is what these paths risk, so
every configuration runs its full sequence: config 2 and the f32 path on all 512 rows,
configs 3 and 4 on 65 rows spanning every batch tile (every 8th row and the last; the
oracle costs 3.7 / 14.7 MFLOP per row-step there), config 5's 4096 variable-length rows on
one GPU on 256 rows spanning every length-sorted tile, with every masked output checked
for exact zeros.  Tolerances are the north star's (16-bit: max 2e-2, mean 5e-3; f32: max
1e-4).  Set PLSTM_PARITY_LOG to a file path to append each case's errors as a JSON line.
"""
from __future__ import annotations

import json
import os

import numpy as np
import pytest
import torch

from helpers import TOL16_MAX, TOL16_MEAN, TOL32_MAX, make_model, oracle_of, weights_of
from persistent_lstm_hip_b200 import core

pytestmark = pytest.mark.gpu

B, T, I, L, O = 512, 1000, 5, 4, 24


def _x(B_, dtype, dev, seed=1):
    return torch.randn(B_, T, I, generator=torch.Generator().manual_seed(seed)).to(dev, dtype)


def _errors(got, ref):
    g = got.detach().to("cpu", torch.float64).numpy()
    d = np.abs(g - ref)
    assert np.isfinite(g).all()
    return float(d.max()), float(d.mean())


def _check(case, pairs, tol_max, tol_mean=None):
    """pairs: (name, device tensor, oracle array); asserts and logs the errors."""
    rec = {"case": case}
    bad = []
    for name, got, ref in pairs:
        mx, mean = _errors(got, ref)
        rec[name] = {"max_abs": mx, "mean_abs": mean}
        if mx > tol_max or (tol_mean is not None and mean > tol_mean):
            bad.append(f"{name}: max {mx:.3g} mean {mean:.3g}")
    path = os.environ.get("PLSTM_PARITY_LOG")
    if path:
        with open(path, "a") as f:
            f.write(json.dumps(rec) + "\n")
    print(json.dumps(rec))
    assert not bad, f"{case}: " + "; ".join(bad)


@pytest.mark.parametrize("mode", ["last", "seq"])
def test_cfg2_all_rows(cuda_device, mode):
    """Config 2 (H = 128, f16), every one of the 512 rows: out, h_n and c_n."""
    H = 128
    w = weights_of(make_model(I, H, L, O, seed=0), L, torch.float16, cuda_device)
    x = _x(B, torch.float16, cuda_device)
    pw = core.PackedWeights(*w, out_mode=mode)
    assert pw.backend == "tc"
    out, h_n, c_n = pw.forward(x, check=True, c_n_f32=True)
    r_out, r_h, r_c = oracle_of(x, *w, out_mode=mode)
    _check(f"cfg2 f16 {mode} all 512 rows", [("out", out, r_out), ("h_n", h_n, r_h), ("c_n", c_n, r_c)],
           TOL16_MAX, TOL16_MEAN)


def test_f32_cfg2_shape_all_rows(cuda_device):
    """The f32 path at the config-2 shape (B = 512, T = 1000): every output of every step of
    every row within the north star's 1e-4."""
    H = 128
    w = weights_of(make_model(I, H, L, O, seed=0), L, torch.float32, cuda_device)
    x = _x(B, torch.float32, cuda_device)
    pw = core.PackedWeights(*w, out_mode="seq")
    assert pw.backend == "simt"
    out, h_n, c_n = pw.forward(x, check=True)
    r_out, r_h, r_c = oracle_of(x, *w, out_mode="seq")
    _check("f32 cfg2-shape seq all 512 rows", [("out", out, r_out), ("h_n", h_n, r_h), ("c_n", c_n, r_c)],
           TOL32_MAX)


@pytest.mark.parametrize("H, dtype, name", [(256, torch.float16, "cfg3"), (512, torch.bfloat16, "cfg4")])
def test_cfg3_cfg4_sampled_rows(cuda_device, H, dtype, name):
    """Configs 3 (H = 256, f16) and 4 (H = 512, bf16), B = 512, T = 1000, [B, O] (the layer
    path); 65 rows spanning every batch tile, with h_n and c_n of every layer."""
    w = weights_of(make_model(I, H, L, O, seed=0), L, dtype, cuda_device)
    x = _x(B, dtype, cuda_device)
    pw = core.PackedWeights(*w, out_mode="last")
    assert pw.backend == "tc"
    out, h_n, c_n = pw.forward(x, check=True, c_n_f32=True)
    rows = np.unique(np.r_[np.arange(0, B, 8), B - 1])
    r_out, r_h, r_c = oracle_of(x, *w, out_mode="last", rows=rows)
    _check(f"{name} H{H} {str(dtype)[6:]} last, {rows.size} rows",
           [("out", out[rows], r_out), ("h_n", h_n[:, rows], r_h), ("c_n", c_n[:, rows], r_c)],
           TOL16_MAX, TOL16_MEAN)


def test_cfg5_4096_rows_one_gpu(cuda_device):
    """Config 5 on one GPU: 4096 rows, lengths uniform in [200, 1000] (seed 2), [B, T, O]
    zero past each length.  256 rows spanning every length-sorted tile (4 per 64 rows of the
    sorted order) against the oracle; every masked output of every row exactly zero."""
    H, Bv = 128, 4096
    w = weights_of(make_model(I, H, L, O, seed=0), L, torch.float16, cuda_device)
    x = _x(Bv, torch.float16, cuda_device, seed=3)
    lens = torch.randint(200, T + 1, (Bv,), generator=torch.Generator().manual_seed(2), dtype=torch.int32)
    pw = core.PackedWeights(*w, out_mode="seq")
    out, h_n, c_n = pw.forward(x, lengths=lens.to(cuda_device), check=True, c_n_f32=True)
    steps = torch.arange(T, device=cuda_device)[None, :]
    masked = steps >= lens.to(cuda_device)[:, None]
    assert int(out[masked].ne(0).sum()) == 0, "outputs past a row's length must be exactly zero"
    order = torch.sort(lens, descending=True, stable=True).indices.numpy()
    rows = np.sort(np.r_[order[0::64], order[1::64], order[31::64], order[63::64]])
    r_out, r_h, r_c = oracle_of(x, *w, lengths=lens, out_mode="seq", rows=rows)
    _check(f"cfg5 f16 seq varlen 4096 rows, {rows.size} sampled",
           [("out", out[rows], r_out), ("h_n", h_n[:, rows], r_h), ("c_n", c_n[:, rows], r_c)],
           TOL16_MAX, TOL16_MEAN)
