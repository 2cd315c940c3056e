"""plstm_forward_packed_noalloc: the forward for callers that cannot give the
library a device workspace (a plugin host whose execute hook must not allocate,
or a program on a fixed device-memory budget).  It runs the same kernels on the
same tiles as the workspace entry point, so its results must be bit-identical to
that entry point's, call after call, although every call reuses the same
library-held scratch array with whatever the previous call left in it.  This file
is collected last on purpose."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from helpers import assert_close16, make_model, oracle_of, weights_of
from persistent_lstm_hip_b200 import _lib, core

pytestmark = pytest.mark.gpu

I, H, L, O = 5, 128, 4, 24


def _stream():
    return torch.cuda.current_stream().cuda_stream


def _model(dev, dtype=torch.float16, seed=21):
    return weights_of(make_model(I, H, L, O, seed=seed), L, dtype, dev)


def _problem(dev, B, T, varlen, dtype=torch.float16, seed=5):
    x = torch.randn(B, T, I, generator=torch.Generator().manual_seed(seed)).to(dev, dtype)
    lens = None
    if varlen:
        g = torch.Generator().manual_seed(seed + 1)
        lens = torch.randint(max(1, T // 5), T + 1, (B,), generator=g, dtype=torch.int32).to(dev)
    return x, lens


def _call_noalloc(pw, x, lens, like):
    """One no-allocation forward; outputs start as NaN so that a row it skips shows."""
    B, T = int(x.shape[0]), int(x.shape[1])
    d = pw.desc(batch=B, seq_len=T, extra_flags=_lib.FLAG_SYNC_CHECK)
    got = [torch.full_like(t, float("nan")) for t in like]
    rc = _lib.load().plstm_forward_packed_noalloc(
        ctypes.byref(d), pw.blob.data_ptr(), x.data_ptr(), None if lens is None else lens.data_ptr(), None, None,
        got[0].data_ptr(), got[1].data_ptr(), got[2].data_ptr(), _stream())
    _lib.check(rc)
    torch.cuda.synchronize()
    return got


def _assert_equal(got, ref, what):
    for name, g, r in zip(("out", "h_n", "c_n"), got, ref):
        assert torch.equal(g, r), f"{what} {name}: differs from the workspace entry point " \
                                  f"(max |d| = {(g.double() - r.double()).abs().max().item():.3g})"


@pytest.mark.parametrize("mode, varlen", [("last", False), ("seq", True), ("hseq", True)])
def test_noalloc_matches_workspace_entry_twice(cuda_device, mode, varlen):
    w = _model(cuda_device)
    pw = core.PackedWeights(*w, out_mode=mode, backend="tc")
    x, lens = _problem(cuda_device, 96, 40, varlen)
    ref = pw.forward(x, lengths=lens, check=True)
    for call in range(2):  # the second call reuses the scratch the first one left behind
        got = _call_noalloc(pw, x, lens, ref)
        _assert_equal(got, ref, f"call {call}")
    rows = np.arange(0, 96, 7)
    r_out, r_h, r_c = oracle_of(x, *w, lengths=None if lens is None else lens.cpu(), out_mode=mode, rows=rows)
    assert_close16(got[0][rows], r_out, "out vs oracle")
    assert_close16(got[1][:, rows], r_h, "h_n vs oracle")
    assert_close16(got[2][:, rows], r_c, "c_n vs oracle")


def test_noalloc_sequence_of_different_problems(cuda_device):
    """Calls of different sizes one after the other: a large variable-length batch whose
    32-row tiles need a second wave (both tile heights are enqueued and one is chosen on
    the device), then smaller fixed- and variable-length batches, then the large one
    again.  Each must equal its own workspace-path result although the array holds the
    previous, larger problem's tiles, permutation and lengths."""
    w = _model(cuda_device, seed=23)
    cases = [(900, 400, True, "seq"), (64, 40, False, "last"), (200, 120, True, "hseq"), (33, 7, True, "last"),
             (900, 400, True, "seq")]
    pws = {m: core.PackedWeights(*w, out_mode=m, backend="tc") for m in ("seq", "last", "hseq")}
    inputs, refs = [], []
    for i, (B, T, varlen, mode) in enumerate(cases):
        x, lens = _problem(cuda_device, B, T, varlen, seed=30 + (i % 4))
        inputs.append((x, lens))
        refs.append(pws[mode].forward(x, lengths=lens, check=True))
    for i, ((B, T, varlen, mode), (x, lens), ref) in enumerate(zip(cases, inputs, refs)):
        got = _call_noalloc(pws[mode], x, lens, ref)
        _assert_equal(got, ref, f"call {i} (B={B}, T={T}, {mode})")
    # The large variable-length call against the oracle on rows from the first and last tiles.
    x, lens = inputs[-1]
    rows = np.array([0, 1, 31, 32, 450, 867, 898, 899])
    r_out, r_h, _ = oracle_of(x, *w, lengths=lens.cpu(), out_mode="seq", rows=rows)
    assert_close16(got[0][rows], r_out, "B=900 out vs oracle")
    assert_close16(got[1][:, rows], r_h, "B=900 h_n vs oracle")


def test_noalloc_bf16(cuda_device):
    w = _model(cuda_device, dtype=torch.bfloat16, seed=24)
    pw = core.PackedWeights(*w, out_mode="seq", backend="tc")
    x, lens = _problem(cuda_device, 40, 30, True, dtype=torch.bfloat16)
    ref = pw.forward(x, lengths=lens, check=True)
    _assert_equal(_call_noalloc(pw, x, lens, ref), ref, "bf16")


def test_noalloc_rejects_problems_beyond_its_scratch(cuda_device):
    pw = core.PackedWeights(*_model(cuda_device, seed=22), out_mode="last", backend="tc")
    d = pw.desc(batch=8192, seq_len=4000)
    rc = _lib.load().plstm_forward_packed_noalloc(ctypes.byref(d), pw.blob.data_ptr(), 16, None, None, None, 16,
                                                  None, None, _stream())
    assert rc == _lib.EINVAL
    assert "24 MiB" in _lib.last_error()


def test_noalloc_keeps_the_callers_device(cuda_device):
    pw = core.PackedWeights(*_model(cuda_device), out_mode="last", backend="tc")
    x, _ = _problem(cuda_device, 16, 8, False)
    ref = pw.forward(x, check=True)
    before = torch.cuda.current_device()
    _call_noalloc(pw, x, None, ref)
    assert torch.cuda.current_device() == before
