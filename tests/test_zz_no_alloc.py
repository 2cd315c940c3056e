"""plstm_forward_packed_noalloc: the forward for callers that cannot give the
library a device workspace (a plugin host whose execute hook must not allocate,
or a program on a fixed device-memory budget).  It must match the workspace
entry point, call after call, although every call reuses the same library-held
scratch array.  This file is collected last on purpose."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from helpers import TOL16_MAX, TOL16_MEAN, make_model, weights_of
from persistent_lstm_hip_b200 import _lib, core

pytestmark = pytest.mark.gpu


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _reference_and_desc(dev, B, T, mode, varlen):
    I, H, L, O = 5, 128, 4, 24
    m = make_model(I, H, L, O, seed=21)
    w = weights_of(m, L, torch.float16, dev)
    pw = core.PackedWeights(*w, out_mode=mode, backend="tc")
    x = torch.randn(B, T, I, generator=torch.Generator().manual_seed(5)).to(dev, torch.float16)
    lens = None
    if varlen:
        lens = torch.randint(1, T + 1, (B,), generator=torch.Generator().manual_seed(6), dtype=torch.int32).to(dev)
    ref_out, ref_h, ref_c = pw.forward(x, lengths=lens, check=True)
    return pw, x, lens, (ref_out, ref_h, ref_c)


def _call_noalloc(pw, x, lens, shapes, check=True):
    B, T = int(x.shape[0]), int(x.shape[1])
    d = pw.desc(batch=B, seq_len=T, extra_flags=_lib.FLAG_SYNC_CHECK if check else 0)
    out = torch.full(shapes[0], float("nan"), dtype=torch.float16, device=x.device)
    h_n = torch.full(shapes[1], float("nan"), dtype=torch.float16, device=x.device)
    c_n = torch.full(shapes[2], float("nan"), dtype=torch.float16, device=x.device)
    rc = _lib.load().plstm_forward_packed_noalloc(
        ctypes.byref(d), pw.blob.data_ptr(), x.data_ptr(), None if lens is None else lens.data_ptr(), None, None,
        out.data_ptr(), h_n.data_ptr(), c_n.data_ptr(), _stream())
    _lib.check(rc)
    torch.cuda.synchronize()
    return out, h_n, c_n


def _close(got, ref, what):
    g = got.double().cpu().numpy()
    r = ref.double().cpu().numpy()
    d = np.abs(g - r)
    assert np.isfinite(g).all(), f"{what}: non-finite values"
    assert d.max() <= TOL16_MAX and d.mean() <= TOL16_MEAN, f"{what}: max {d.max():.3g} mean {d.mean():.3g}"


@pytest.mark.parametrize("mode, varlen", [("last", False), ("seq", True)])
def test_noalloc_matches_workspace_entry_twice(cuda_device, mode, varlen):
    pw, x, lens, ref = _reference_and_desc(cuda_device, 96, 40, mode, varlen)
    shapes = [tuple(t.shape) for t in ref]
    for call in range(2):  # the second call reuses the scratch the first one left behind
        got = _call_noalloc(pw, x, lens, shapes)
        for name, g, r in zip(("out", "h_n", "c_n"), got, ref):
            _close(g, r, f"call {call} {name}")


def test_noalloc_rejects_problems_beyond_its_scratch(cuda_device):
    I, H, L, O = 5, 128, 4, 24
    m = make_model(I, H, L, O, seed=22)
    pw = core.PackedWeights(*weights_of(m, L, torch.float16, cuda_device), out_mode="last", backend="tc")
    d = pw.desc(batch=8192, seq_len=4000)
    rc = _lib.load().plstm_forward_packed_noalloc(ctypes.byref(d), pw.blob.data_ptr(), 16, None, None, None, 16,
                                                  None, None, _stream())
    assert rc == _lib.EINVAL
    assert "24 MiB" in _lib.last_error()
