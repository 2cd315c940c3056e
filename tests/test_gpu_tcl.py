"""GPU parity of the layer-sequential tensor-core path (any hidden size up to 512; per layer a
tcgen05 projection GEMM and a cluster recurrence with W_hh resident in tensor
memory) against the f64 oracle, with the north star's 16-bit tolerances."""
from __future__ import annotations

import pytest
import torch

from helpers import assert_close16, make_model, oracle_of, weights_of
import persistent_lstm_hip_b200 as plstm
from persistent_lstm_hip_b200 import core

pytestmark = pytest.mark.gpu


def _x(B, T, I, dtype, dev, seed=1):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(B, T, I, generator=g).to(device=dev, dtype=dtype)


@pytest.mark.parametrize("H", [256, 512])
@pytest.mark.parametrize("B, T, L", [(1, 1, 1), (5, 7, 2), (70, 12, 3)])
@pytest.mark.parametrize("mode", ["seq", "last", "hseq"])
def test_tcl_matches_oracle(cuda_device, H, B, T, L, mode):
    I, O = 5, 24
    dtype = torch.float16 if H == 256 else torch.bfloat16
    m = make_model(I, H, L, O, seed=H + L)
    w = weights_of(m, L, dtype, cuda_device)
    x = _x(B, T, I, dtype, cuda_device, seed=B + T)
    pw = core.PackedWeights(*w, out_mode=mode, backend="tc")
    assert pw.backend == "tc"
    out, h_n, c_n = pw.forward(x, check=True)
    r_out, r_h, r_c = oracle_of(x, *w, out_mode=mode)
    assert_close16(out, r_out, "out")
    assert_close16(h_n, r_h, "h_n")
    assert_close16(c_n, r_c, "c_n")


@pytest.mark.parametrize("H, dtype", [(256, torch.bfloat16), (512, torch.float16)])
@pytest.mark.parametrize("mode", ["seq", "last"])
def test_tcl_varlen_and_state(cuda_device, H, dtype, mode):
    B, T, I, L, O = 67, 16, 5, 2, 24
    m = make_model(I, H, L, O, seed=11)
    w = weights_of(m, L, dtype, cuda_device)
    x = _x(B, T, I, dtype, cuda_device)
    g = torch.Generator().manual_seed(3)
    lens = torch.randint(0, T + 1, (B,), generator=g, dtype=torch.int32)
    lens[0] = T
    hx = ((0.5 * torch.randn(L, B, H, generator=g)).to(cuda_device, dtype),
          (0.5 * torch.randn(L, B, H, generator=g)).to(cuda_device, dtype))
    pw = core.PackedWeights(*w, out_mode=mode, backend="tc")
    out, h_n, c_n = pw.forward(x, lengths=lens.to(cuda_device), hx=hx, check=True)
    r_out, r_h, r_c = oracle_of(x, *w, lengths=lens, hx=hx, out_mode=mode)
    assert_close16(out, r_out, "out")
    assert_close16(h_n, r_h, "h_n")
    assert_close16(c_n, r_c, "c_n")
    if mode == "seq":
        o = out.cpu()
        for b in range(B):
            assert torch.all(o[b, int(lens[b]):] == 0)


def test_tcl_is_the_auto_backend_and_matches_simt(cuda_device):
    """The default backend for H = 256 is the tensor-core path; it agrees with the
    FFMA backend on the same 16-bit weights."""
    B, T, I, H, L, O = 9, 20, 5, 256, 2, 24
    m = make_model(I, H, L, O, seed=2)
    w = weights_of(m, L, torch.float16, cuda_device)
    x = _x(B, T, I, torch.float16, cuda_device)
    assert core.PackedWeights(*w, out_mode="last").backend == "tc"
    a, _, _ = plstm.lstm_linear_forward(x, *w, out_mode="last", check=True)
    b, _, _ = plstm.lstm_linear_forward(x, *w, out_mode="last", backend="simt", check=True)
    assert (a.float() - b.float()).abs().max().item() <= 2e-2


# Generic hidden sizes: every multiple of 64 up to 512 runs on the layer-sequential
# tensor-core path (C = H / 32 CTAs per cluster, 2..16), as does H = 128 outside the
# wavefront kernel's envelope (more than 8 layers, or a Linear head wider than 32).
@pytest.mark.parametrize("H", [64, 192, 320, 384, 448])
@pytest.mark.parametrize("mode", ["seq", "last", "hseq"])
def test_tcl_generic_hidden_sizes(cuda_device, H, mode):
    B, T, I, L, O = 70, 11, 5, 2, 24
    dtype = torch.bfloat16 if H in (192, 448) else torch.float16
    m = make_model(I, H, L, O, seed=H)
    w = weights_of(m, L, dtype, cuda_device)
    x = _x(B, T, I, dtype, cuda_device, seed=H + 1)
    pw = core.PackedWeights(*w, out_mode=mode, backend="tc")
    assert pw.backend == "tc"
    out, h_n, c_n = pw.forward(x, check=True)
    r_out, r_h, r_c = oracle_of(x, *w, out_mode=mode)
    assert_close16(out, r_out, "out")
    assert_close16(h_n, r_h, "h_n")
    assert_close16(c_n, r_c, "c_n")


@pytest.mark.parametrize("H", [64, 384])
def test_tcl_generic_varlen_and_state(cuda_device, H):
    B, T, I, L, O = 45, 14, 5, 3, 24
    m = make_model(I, H, L, O, seed=H + 7)
    w = weights_of(m, L, torch.float16, cuda_device)
    x = _x(B, T, I, torch.float16, cuda_device)
    g = torch.Generator().manual_seed(4)
    lens = torch.randint(0, T + 1, (B,), generator=g, dtype=torch.int32)
    lens[0] = T
    hx = ((0.5 * torch.randn(L, B, H, generator=g)).to(cuda_device, torch.float16),
          (0.5 * torch.randn(L, B, H, generator=g)).to(cuda_device, torch.float16))
    pw = core.PackedWeights(*w, out_mode="seq", backend="tc")
    out, h_n, c_n = pw.forward(x, lengths=lens.to(cuda_device), hx=hx, check=True)
    r_out, r_h, r_c = oracle_of(x, *w, lengths=lens, hx=hx, out_mode="seq")
    assert_close16(out, r_out, "out")
    assert_close16(h_n, r_h, "h_n")
    assert_close16(c_n, r_c, "c_n")


@pytest.mark.parametrize("L, O", [(10, 24), (2, 40)])
def test_tcl_h128_outside_wavefront_envelope(cuda_device, L, O):
    B, T, I, H = 33, 9, 5, 128
    m = make_model(I, H, L, O, seed=L + O)
    w = weights_of(m, L, torch.float16, cuda_device)
    x = _x(B, T, I, torch.float16, cuda_device, seed=L)
    pw = core.PackedWeights(*w, out_mode="seq", backend="tc")
    assert pw.backend == "tc"
    out, h_n, c_n = pw.forward(x, check=True)
    r_out, r_h, r_c = oracle_of(x, *w, out_mode="seq")
    assert_close16(out, r_out, "out")
    assert_close16(h_n, r_h, "h_n")
    assert_close16(c_n, r_c, "c_n")


def test_tcl_rejects_other_hidden_sizes(cuda_device):
    for H in (513, 640, 1024):
        assert core.select_backend(input_size=5, hidden_size=H, num_layers=2, output_size=24,
                                   dtype=torch.float16, device=cuda_device.index or 0) == "simt"


# Any hidden size up to 512 runs on the layer path, zero-padded to the next multiple of 64.
@pytest.mark.parametrize("H, L", [(150, 2), (200, 3), (300, 2), (500, 1), (100, 10)])
def test_tcl_padded_hidden_sizes(cuda_device, H, L):
    B, T, I, O = 41, 10, 5, 24
    m = make_model(I, H, L, O, seed=H + L)
    w = weights_of(m, L, torch.float16, cuda_device)
    x = _x(B, T, I, torch.float16, cuda_device, seed=H)
    g = torch.Generator().manual_seed(H)
    lens = torch.randint(0, T + 1, (B,), generator=g, dtype=torch.int32)
    lens[0] = T
    hx = ((0.5 * torch.randn(L, B, H, generator=g)).to(cuda_device, torch.float16),
          (0.5 * torch.randn(L, B, H, generator=g)).to(cuda_device, torch.float16))
    for mode in ("seq", "last", "hseq"):
        pw = core.PackedWeights(*w, out_mode=mode, backend="tc")
        assert pw.backend == "tc"
        out, h_n, c_n = pw.forward(x, lengths=lens.to(cuda_device), hx=hx, check=True)
        r_out, r_h, r_c = oracle_of(x, *w, lengths=lens, hx=hx, out_mode=mode)
        assert_close16(out, r_out, f"{mode} out")
        assert_close16(h_n, r_h, f"{mode} h_n")
        assert_close16(c_n, r_c, f"{mode} c_n")


# Layer-0 inputs up to 128 columns (the projection's K = I rounded up to 16).
@pytest.mark.parametrize("H, I", [(256, 17), (192, 64), (512, 100), (256, 128), (128, 48)])
def test_tcl_wide_inputs(cuda_device, H, I):
    B, T, O = 39, 9, 24
    L = 9 if H == 128 else 2  # H = 128 takes the layer path beyond 8 layers
    m = make_model(I, H, L, O, seed=H + I)
    w = weights_of(m, L, torch.bfloat16, cuda_device)
    x = _x(B, T, I, torch.bfloat16, cuda_device, seed=I)
    for mode in ("seq", "last"):
        pw = core.PackedWeights(*w, out_mode=mode, backend="tc")
        assert pw.backend == "tc"
        out, h_n, c_n = pw.forward(x, check=True)
        r_out, r_h, r_c = oracle_of(x, *w, out_mode=mode)
        assert_close16(out, r_out, f"{mode} out")
        assert_close16(h_n, r_h, f"{mode} h_n")
        assert_close16(c_n, r_c, f"{mode} c_n")


# Batches whose 64-row tiles need a second wave of 12..16-CTA clusters run 80-row tiles.
@pytest.mark.parametrize("H", [384, 448, 512])
def test_tcl_80_row_tiles(cuda_device, H):
    B, T, I, L, O = 520, 5, 5, 2, 24
    m = make_model(I, H, L, O, seed=H + 3)
    w = weights_of(m, L, torch.bfloat16, cuda_device)
    x = _x(B, T, I, torch.bfloat16, cuda_device, seed=H)
    g = torch.Generator().manual_seed(H + 1)
    lens = torch.randint(0, T + 1, (B,), generator=g, dtype=torch.int32)
    lens[0] = T
    hx = ((0.5 * torch.randn(L, B, H, generator=g)).to(cuda_device, torch.bfloat16),
          (0.5 * torch.randn(L, B, H, generator=g)).to(cuda_device, torch.bfloat16))
    for mode, kw in (("seq", {"lengths": lens.to(cuda_device), "hx": hx}), ("last", {})):
        pw = core.PackedWeights(*w, out_mode=mode, backend="tc")
        out, h_n, c_n = pw.forward(x, check=True, **kw)
        okw = {"lengths": lens, "hx": hx} if kw else {}
        r_out, r_h, r_c = oracle_of(x, *w, out_mode=mode, **okw)
        assert_close16(out, r_out, f"{mode} out")
        assert_close16(h_n, r_h, f"{mode} h_n")
        assert_close16(c_n, r_c, f"{mode} c_n")


# Every tile height (PLSTM_TCL_NT forces one the hidden size has): 32 / 48 / 64 rows for
# H <= 256, 64 / 80 for H >= 384; the automatic choice is the smallest that runs the batch
# in one wave of clusters.
@pytest.mark.parametrize("H, L, nt", [(256, 2, 32), (256, 2, 48), (256, 2, 64), (64, 3, 48), (128, 9, 32),
                                      (512, 2, 64), (512, 2, 80), (448, 1, 80)])
def test_tcl_tile_heights(cuda_device, monkeypatch, H, L, nt):
    monkeypatch.setenv("PLSTM_TCL_NT", str(nt))
    B, T, I, O = 171, 4, 5, 24
    m = make_model(I, H, L, O, seed=H + nt)
    w = weights_of(m, L, torch.float16, cuda_device)
    x = _x(B, T, I, torch.float16, cuda_device, seed=nt)
    g = torch.Generator().manual_seed(nt)
    lens = torch.randint(0, T + 1, (B,), generator=g, dtype=torch.int32)
    lens[0] = T
    for mode in ("seq", "last", "hseq"):
        pw = core.PackedWeights(*w, out_mode=mode, backend="tc")
        out, h_n, c_n = pw.forward(x, lengths=lens.to(cuda_device), check=True)
        r_out, r_h, r_c = oracle_of(x, *w, lengths=lens, out_mode=mode)
        assert_close16(out, r_out, f"{mode} out")
        assert_close16(h_n, r_h, f"{mode} h_n")
        assert_close16(c_n, r_c, f"{mode} c_n")
