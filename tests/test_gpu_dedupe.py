"""Duplicate-row elimination (PLSTM_FLAG_DEDUPE, plstm_unique_rows).

The reference computes an all-rows-identical batch once and broadcasts it
(persistent_lstm_hip/persistent_lstm_hip/model.py:493-530).  The general form
here groups any identical rows on the GPU; these tests check the grouping
against the oracle's restatement and that a deduplicated forward returns,
bit for bit, what the full forward returns (every row's arithmetic is
independent of the other rows), which in turn is checked against the oracle.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

import persistent_lstm_hip_b200 as P
from oracle import oracle
from persistent_lstm_hip_b200 import _lib, core

from helpers import assert_close16, make_model, oracle_of, weights_of

pytestmark = pytest.mark.gpu


def _rows_with_duplicates(B, T, I, distinct, dtype, seed):
    g = torch.Generator().manual_seed(seed)
    base = torch.randn(distinct, T, I, generator=g)
    pick = torch.randint(0, distinct, (B,), generator=g)
    return base[pick].to(dtype).cuda(), pick


def _np(t):
    return t.detach().cpu().numpy()


def _check_grouping(x, lengths=None, hx=None):
    row_map, uniq, count = P.unique_rows(x, lengths=lengths, hx=hx)
    h0 = c0 = None
    if hx is not None:
        h0, c0 = _np(hx[0].view(torch.int16)), _np(hx[1].view(torch.int16))
    xb = _np(x.view(torch.int16)) if x.element_size() == 2 else _np(x.view(torch.int32))
    ref_map, ref_first, ref_count = oracle.unique_rows(
        xb, lengths=None if lengths is None else _np(lengths), h0=h0, c0=c0)
    assert count == ref_count
    np.testing.assert_array_equal(_np(row_map), ref_map)
    np.testing.assert_array_equal(_np(uniq), ref_first)
    return count


def test_unique_rows_plain():
    x, pick = _rows_with_duplicates(96, 33, 5, 7, torch.float16, 1)
    assert _check_grouping(x) == len(set(pick.tolist()))


def test_unique_rows_all_equal_and_all_distinct():
    x = torch.randn(1, 40, 5).half().cuda().expand(64, 40, 5).contiguous()
    assert _check_grouping(x) == 1
    y = torch.randn(64, 40, 5).half().cuda()
    assert _check_grouping(y) == 64


def test_unique_rows_lengths_ignore_padding():
    x, _ = _rows_with_duplicates(80, 50, 3, 5, torch.bfloat16, 2)
    g = torch.Generator().manual_seed(3)
    lengths = torch.randint(1, 51, (5,), generator=g)[torch.randint(0, 5, (80,), generator=g)]
    # Scribble past every row's length: padding must not split a group.
    for b in range(80):
        x[b, int(lengths[b]):] = torch.randn(50 - int(lengths[b]), 3, generator=g).to(torch.bfloat16).cuda()
    _check_grouping(x, lengths=lengths.cuda())


def test_unique_rows_hx_and_f32():
    x, _ = _rows_with_duplicates(40, 12, 4, 3, torch.float32, 4)
    x[7] = x[8]
    h0 = torch.zeros(2, 40, 16, device="cuda")
    c0 = torch.zeros(2, 40, 16, device="cuda")
    c0[1, 7, 3] = 0.5  # row 7 now differs from its x-duplicates
    _check_grouping(x, hx=(h0, c0))
    row_map, _, _ = P.unique_rows(x, hx=(h0, c0))
    assert int((row_map == row_map[7]).sum()) == 1
    plain, _, _ = P.unique_rows(x)
    assert plain[7] == plain[8]


def _forward_pair(x, weights, **kw):
    a = core.lstm_linear_forward(x, *weights, **kw)
    b = core.lstm_linear_forward(x, *weights, dedupe=True, **kw)
    return a, b


def _assert_same(a, b):
    for u, v in zip(a, b):
        if u is None:
            assert v is None
            continue
        assert torch.equal(u, v), (u.float() - v.float()).abs().max().item()


@pytest.mark.parametrize("out_mode", ["seq", "last"])
def test_dedupe_forward_h128_tensor_core(out_mode):
    B, T, I, H, L, O = 200, 48, 5, 128, 4, 24
    m = make_model(I, H, L, O, seed=21)
    wts = weights_of(m, L, torch.float16, "cuda")
    x, pick = _rows_with_duplicates(B, T, I, 9, torch.float16, 22)
    a, b = _forward_pair(x, wts, out_mode=out_mode, backend="tc")
    _assert_same(a, b)
    rows = sorted(set(int(i) for i in torch.unique(pick)))
    first = [int((pick == r).nonzero()[0]) for r in rows]
    ref = oracle_of(x, *wts, out_mode=out_mode, rows=first)
    assert_close16(b[0][first], ref[0], "out")
    assert_close16(b[1][:, first], ref[1], "h_n")


def test_dedupe_forward_varlen_hx_h256():
    B, T, I, H, L, O = 72, 40, 5, 256, 2, 8
    m = make_model(I, H, L, O, seed=23)
    wts = weights_of(m, L, torch.float16, "cuda")
    x, pick = _rows_with_duplicates(B, T, I, 6, torch.float16, 24)
    lengths = (10 + 5 * pick).to(torch.int32)
    lengths[0] = T
    g = torch.Generator().manual_seed(25)
    h0 = (0.3 * torch.randn(L, 6, H, generator=g))[:, pick].half().cuda()
    c0 = (0.3 * torch.randn(L, 6, H, generator=g))[:, pick].half().cuda()
    h0[:, 5] += 0.25  # row 5 stands alone
    a, b = _forward_pair(x, wts, lengths=lengths.cuda(), hx=(h0, c0), out_mode="seq")
    _assert_same(a, b)
    ref = oracle_of(x, *wts, lengths=lengths, hx=(h0, c0), out_mode="seq")
    assert_close16(b[0], ref[0], "out")
    assert_close16(b[2], ref[2], "c_n")


def test_dedupe_forward_simt_f32_hseq():
    B, T, I, H, L = 48, 20, 7, 40, 3
    m = make_model(I, H, L, 4, seed=26)
    wts = weights_of(m, L, torch.float32, "cuda")
    x, _ = _rows_with_duplicates(B, T, I, 4, torch.float32, 27)
    a, b = _forward_pair(x, wts[:4], out_mode="hseq")
    _assert_same(a, b)


def test_dedupe_f32_keeps_the_full_batch_kernel():
    # 700 rows run the L2-streaming FFMA kernel; their 40 distinct rows alone would fit the
    # cluster kernel, whose per-row summation order differs.  The deduplicated forward keeps
    # the full batch's kernel, so the results stay bit-identical.
    B, T, I, H, L, O = 700, 12, 5, 64, 2, 6
    m = make_model(I, H, L, O, seed=32)
    wts = weights_of(m, L, torch.float32, "cuda")
    x, pick = _rows_with_duplicates(B, T, I, 40, torch.float32, 33)
    a, b = _forward_pair(x, wts, out_mode="seq")
    _assert_same(a, b)
    rows = sorted(set(int(i) for i in torch.unique(pick)))[:6]
    first = [int((pick == r).nonzero()[0]) for r in rows]
    ref = oracle_of(x, *wts, out_mode="seq", rows=first)
    assert (b[0][first].double().cpu() - torch.from_numpy(ref[0])).abs().max() <= 1e-4


def test_dedupe_no_duplicates_and_uniform():
    B, T, I, H, L, O = 64, 30, 5, 128, 4, 24
    m = make_model(I, H, L, O, seed=28)
    wts = weights_of(m, L, torch.float16, "cuda")
    x = torch.randn(B, T, I).half().cuda()
    _assert_same(*_forward_pair(x, wts, out_mode="last"))
    xu = x[:1].expand(B, T, I).contiguous()
    a, b = _forward_pair(xu, wts, out_mode="last")
    _assert_same(a, b)
    assert torch.equal(b[0], b[0][:1].expand_as(b[0]))


def test_dedupe_regressor_env(monkeypatch):
    B, T, I, H, L, O = 128, 25, 5, 128, 4, 24
    m = make_model(I, H, L, O, seed=29).half().cuda()
    reg = P.convert_regressor_module(m)
    x, _ = _rows_with_duplicates(B, T, I, 3, torch.float16, 30)
    monkeypatch.setenv("PERSISTENT_LSTM_HIP_UNIFORM_BATCH", "0")
    plain = reg(x)
    monkeypatch.setenv("PERSISTENT_LSTM_HIP_UNIFORM_BATCH", "dedupe")
    assert torch.equal(reg(x), plain)


def test_dedupe_refused_under_capture():
    B, T, I, H, L, O = 16, 8, 5, 128, 4, 24
    m = make_model(I, H, L, O, seed=31)
    wts = weights_of(m, L, torch.float16, "cuda")
    pw = core.PackedWeights(*wts, out_mode="last")
    x = torch.randn(B, T, I).half().cuda()
    pw.forward(x)  # warm the library outside the capture
    graph = torch.cuda.CUDAGraph()
    with pytest.raises(_lib.PlstmError):
        with torch.cuda.graph(graph):
            pw.forward(x, dedupe=True)
    torch.cuda.synchronize()
    out, _, _ = pw.forward(x, dedupe=True)
    ref, _, _ = pw.forward(x)
    assert torch.equal(out, ref)
