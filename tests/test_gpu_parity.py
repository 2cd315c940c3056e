"""GPU parity tests: every CUDA path against the f64 oracle (which is pinned to
the reference's own outputs in test_oracle.py).  Tolerances are the north
star's: 16-bit paths max |err| <= 2e-2 and mean |err| <= 5e-3, f32 path
max |err| <= 1e-4."""
from __future__ import annotations

import ctypes
import os

import numpy as np
import pytest
import torch

from conftest import golden_weights, load_golden
from helpers import (TOL32_MAX, assert_close16, assert_close32, make_model, np64, oracle_of, weights_of)
import persistent_lstm_hip_b200 as plstm
from persistent_lstm_hip_b200 import _lib, core, ext

pytestmark = pytest.mark.gpu


def _rand_x(B, T, I, dtype, dev, seed=1):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(B, T, I, generator=g).to(device=dev, dtype=dtype)


def _rand_lengths(B, T, seed=2, lo=1):
    g = torch.Generator().manual_seed(seed)
    lens = torch.randint(lo, T + 1, (B,), generator=g, dtype=torch.int32)
    lens[0] = T
    return lens


# ---------------------------------------------------------------------------------------
def test_tmem_data_path_layout(cuda_device):
    """tcgen05.ld 16x256b / 32x32b register layouts the wavefront kernel relies on."""
    out = torch.zeros(128 * 24, dtype=torch.int32, device=cuda_device)
    _lib.check(_lib.load().plstm_diag_tmem_layout(out.data_ptr(), torch.cuda.current_stream().cuda_stream))
    got = out.view(4, 32, 24).cpu().numpy().astype(np.int64)
    bad = []
    for w in range(4):
        for t in range(32):
            exp = []
            for base in (32 * w, 32 * w + 16):
                for c in range(2):  # .x2: two 256-bit column chunks
                    for r in range(4):
                        lane = base + t // 4 + (8 if r >= 2 else 0)
                        col = 8 * c + 2 * (t % 4) + (r & 1)
                        exp.append((lane << 8) | col)
            exp += [((32 * w + t) << 8) | (8 + i) for i in range(8)]
            if list(got[w, t]) != exp:
                bad.append((w, t, [hex(v) for v in got[w, t]], [hex(v) for v in exp]))
    assert not bad, f"{len(bad)} threads differ, first: {bad[:2]}"


# ---------------------------------------------------------------------------------------
@pytest.mark.parametrize("mode", ["seq", "last", "hseq"])
@pytest.mark.parametrize("varlen", [False, True])
def test_simt_f32_matches_oracle(cuda_device, mode, varlen):
    B, T, I, H, L, O = 5, 9, 5, 16, 2, 4
    m = make_model(I, H, L, O, seed=3)
    w = weights_of(m, L, torch.float32, cuda_device)
    x = _rand_x(B, T, I, torch.float32, cuda_device)
    lens = _rand_lengths(B, T) if varlen else None
    out, h_n, c_n = plstm.lstm_linear_forward(x, *w, lengths=lens, out_mode=mode, check=True)
    r_out, r_h, r_c = oracle_of(x, *w, lengths=lens, out_mode=mode)
    assert_close32(out, r_out, "out")
    assert_close32(h_n, r_h, "h_n")
    assert_close32(c_n, r_c, "c_n")


def test_simt_f32_with_state_and_golden(cuda_device):
    g = load_golden("ref_state_f64")
    B, T, I, H, L, O = (int(v) for v in g["dims"])
    w_ih, w_hh, b_ih, b_hh, _, _ = golden_weights(g, L)
    f = lambda a: torch.from_numpy(a).to(device=cuda_device, dtype=torch.float32)
    out, h_n, c_n = plstm.lstm_linear_forward(
        f(g["x"]), [f(a) for a in w_ih], [f(a) for a in w_hh], [f(a) for a in b_ih], [f(a) for a in b_hh],
        out_mode="hseq", hx=(f(g["h0"]), f(g["c0"])), check=True)
    assert_close32(out, g["out_h"], "out")
    assert_close32(h_n, g["h_n"], "h_n")
    assert_close32(c_n, g["c_n"], "c_n")


@pytest.mark.parametrize("H, L", [(256, 2), (512, 1), (64, 3)])
def test_simt_16bit_other_hidden_sizes(cuda_device, H, L):
    B, T, I, O = 6, 12, 5, 24
    m = make_model(I, H, L, O, seed=4)
    for dt in (torch.float16, torch.bfloat16):
        w = weights_of(m, L, dt, cuda_device)
        x = _rand_x(B, T, I, dt, cuda_device)
        out, h_n, c_n = plstm.lstm_linear_forward(x, *w, out_mode="seq", backend="simt", check=True)
        r_out, r_h, r_c = oracle_of(x, *w, out_mode="seq")
        assert_close16(out, r_out, f"{dt} out")
        assert_close16(h_n, r_h, f"{dt} h_n")


# The FFMA layer kernel's launch shapes: 1, 2, 4 or 8 batch rows per CTA (by B), the
# [x ; h] contraction split into 1..8 k-slices (by H and K), H above the thread count,
# odd and wide inputs.
@pytest.mark.parametrize("B, T, I, H, L", [(600, 6, 3, 24, 2), (300, 7, 5, 40, 2), (200, 5, 7, 300, 2),
                                           (9, 8, 130, 100, 3), (150, 10, 1, 72, 2)])
def test_simt_f32_launch_shapes(cuda_device, B, T, I, H, L):
    O = 3
    m = make_model(I, H, L, O, seed=5)
    w = weights_of(m, L, torch.float32, cuda_device)
    x = _rand_x(B, T, I, torch.float32, cuda_device, seed=6)
    lens = _rand_lengths(B, T, seed=7)
    g = torch.Generator().manual_seed(8)
    h0 = (0.5 * torch.randn(L, B, H, generator=g)).to(cuda_device)
    c0 = (0.5 * torch.randn(L, B, H, generator=g)).to(cuda_device)
    for mode in ("seq", "hseq"):
        out, h_n, c_n = plstm.lstm_linear_forward(x, *w, lengths=lens, hx=(h0, c0), out_mode=mode, check=True)
        r_out, r_h, r_c = oracle_of(x, *w, lengths=lens, hx=(h0, c0), out_mode=mode)
        assert_close32(out, r_out, f"{mode} out")
        assert_close32(h_n, r_h, "h_n")
        assert_close32(c_n, r_c, "c_n")


# The cluster-resident f32 kernel (H up to 128, I <= 128, batches up to 592 rows): 4, 8 and
# 16 batch rows per 4-CTA cluster, k-slices from 8 to 16, layer-0 inputs of 1 to 128
# columns, hidden sizes that leave padding units in the CTAs (1, 40, 100).
@pytest.mark.parametrize("B, T, I, H, L", [(3, 9, 5, 128, 2), (100, 12, 1, 64, 3), (300, 7, 128, 16, 2),
                                           (592, 5, 17, 112, 2), (150, 10, 40, 32, 1), (40, 8, 3, 100, 2),
                                           (7, 6, 2, 1, 2), (260, 9, 9, 40, 3)])
def test_simt_f32_cluster_kernel(cuda_device, B, T, I, H, L):
    O = 5
    m = make_model(I, H, L, O, seed=11)
    w = weights_of(m, L, torch.float32, cuda_device)
    x = _rand_x(B, T, I, torch.float32, cuda_device, seed=12)
    lens = _rand_lengths(B, T, seed=13, lo=0)
    g = torch.Generator().manual_seed(14)
    h0 = (0.5 * torch.randn(L, B, H, generator=g)).to(cuda_device)
    c0 = (0.5 * torch.randn(L, B, H, generator=g)).to(cuda_device)
    for mode in ("seq", "hseq"):
        out, h_n, c_n = plstm.lstm_linear_forward(x, *w, lengths=lens, hx=(h0, c0), out_mode=mode, check=True)
        r_out, r_h, r_c = oracle_of(x, *w, lengths=lens, hx=(h0, c0), out_mode=mode)
        assert_close32(out, r_out, f"{mode} out")
        assert_close32(h_n, r_h, "h_n")
        assert_close32(c_n, r_c, "c_n")
    # A row's arithmetic does not depend on its cluster companions or the batch size.
    rows = torch.arange(0, B, 3)
    s_out, s_h, s_c = plstm.lstm_linear_forward(x[rows], *w, lengths=lens[rows], hx=(h0[:, rows], c0[:, rows]),
                                                out_mode="hseq")
    assert torch.equal(out[rows], s_out)
    assert torch.equal(h_n[:, rows], s_h)
    assert torch.equal(c_n[:, rows], s_c)


def test_simt_16bit_beyond_tensor_core_hidden(cuda_device):
    B, T, I, H, L, O = 3, 4, 5, 640, 2, 6
    m = make_model(I, H, L, O, seed=9)
    for dt in (torch.float16, torch.bfloat16):
        w = weights_of(m, L, dt, cuda_device)
        x = _rand_x(B, T, I, dt, cuda_device, seed=10)
        out, h_n, c_n = plstm.lstm_linear_forward(x, *w, out_mode="seq", check=True)
        r_out, r_h, r_c = oracle_of(x, *w, out_mode="seq")
        assert_close16(out, r_out, f"{dt} out")
        assert_close16(c_n, r_c, f"{dt} c_n")


# ---------------------------------------------------------------------------------------
TC_SHAPES = [(1, 1, 1), (3, 7, 2), (17, 33, 4), (40, 9, 3), (70, 20, 4)]


@pytest.mark.parametrize("B, T, L", TC_SHAPES)
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("mode", ["seq", "last", "hseq"])
def test_tc_matches_oracle(cuda_device, B, T, L, dtype, mode):
    I, H, O = 5, 128, 24
    m = make_model(I, H, L, O, seed=5 + L)
    w = weights_of(m, L, dtype, cuda_device)
    x = _rand_x(B, T, I, dtype, cuda_device, seed=B + T)
    pw = core.PackedWeights(*w, out_mode=mode, backend="tc")
    assert pw.backend == "tc"
    out, h_n, c_n = pw.forward(x, check=True)
    r_out, r_h, r_c = oracle_of(x, *w, out_mode=mode)
    assert_close16(out, r_out, "out")
    assert_close16(h_n, r_h, "h_n")
    assert_close16(c_n, r_c, "c_n")


@pytest.mark.parametrize("mode", ["seq", "last", "hseq"])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_tc_varlen_and_state(cuda_device, mode, dtype):
    B, T, I, H, L, O = 45, 24, 5, 128, 4, 24
    m = make_model(I, H, L, O, seed=9)
    w = weights_of(m, L, dtype, cuda_device)
    x = _rand_x(B, T, I, dtype, cuda_device)
    lens = _rand_lengths(B, T, lo=0)
    g = torch.Generator().manual_seed(7)
    hx = ((0.5 * torch.randn(L, B, H, generator=g)).to(cuda_device, dtype),
          (0.5 * torch.randn(L, B, H, generator=g)).to(cuda_device, dtype))
    pw = core.PackedWeights(*w, out_mode=mode, backend="tc")
    out, h_n, c_n = pw.forward(x, lengths=lens.to(cuda_device), hx=hx, check=True)
    r_out, r_h, r_c = oracle_of(x, *w, lengths=lens, hx=hx, out_mode=mode)
    assert_close16(out, r_out, "out")
    assert_close16(h_n, r_h, "h_n")
    assert_close16(c_n, r_c, "c_n")
    # Masked positions are exactly zero.
    if mode in ("seq", "hseq"):
        o = out.cpu()
        for b in range(B):
            assert torch.all(o[b, int(lens[b]):] == 0)


def test_tc_equals_simt_bitwise_layouts(cuda_device):
    """All reference weight layouts pack to the same device image."""
    B, T, I, H, L, O = 33, 16, 5, 128, 4, 24
    m = make_model(I, H, L, O, seed=10)
    w_ih, w_hh, b_ih, b_hh, w_lin, b_lin = weights_of(m, L, torch.float16, cuda_device)
    bias = [a + b for a, b in zip(b_ih, b_hh)]
    x = _rand_x(B, T, I, torch.float16, cuda_device)
    from persistent_lstm_hip_b200.packing import pack_recurrent_weight_kpairs as kp
    args_native = [t for l in range(L) for t in (w_ih[l], w_hh[l], bias[l])] + [w_lin, b_lin]
    args_t = [t for l in range(L) for t in (w_ih[l].t().contiguous(), w_hh[l].t().contiguous(), bias[l])] + [w_lin, b_lin]
    args_kp = [t for l in range(L) for t in (kp(w_ih[l]), kp(w_hh[l]), bias[l])] + [w_lin, b_lin]
    args_proj = [t for l in range(L) for t in (w_ih[l], kp(w_hh[l]), bias[l])] + [w_lin, b_lin]
    outs = [ext.persistent_lstm4_forward(x, *args_native),
            ext.persistent_lstm4_forward_packed(x, *args_t),
            ext.persistent_lstm4_forward_interleaved(x, *args_kp),
            ext.persistent_lstm4_forward_monolithic(x, *args_kp),
            ext.persistent_lstm4_forward_projected(x, *args_proj),
            ext.persistent_lstm4_forward_projected_uniform_p4(x, 4, *args_proj),
            ext.persistent_lstm_regressor_forward_generic_projected(x, w_ih, w_hh, bias, w_lin, b_lin)]
    for o in outs[1:]:
        torch.testing.assert_close(o, outs[0], rtol=0, atol=0)
    r_out, _, _ = oracle_of(x, w_ih, w_hh, b_ih, b_hh, w_lin, b_lin, out_mode="last")
    assert_close16(outs[0], r_out, "ext out")
    # The generic kernel agrees with the tensor-core kernel within the 16-bit tolerance.
    simt = core.PackedWeights(w_ih, w_hh, b_ih, b_hh, w_lin, b_lin, out_mode="last", backend="simt")
    assert simt.backend == "simt"
    o_simt, _, _ = simt.forward(x, check=True)
    assert_close16(o_simt, r_out, "simt out")


def test_golden_regressor_through_tc(cuda_device):
    """The reference's own regressor output (f32, H128 L4) reproduced by the f16 kernel."""
    g = load_golden("ref_h128_f32")
    B, T, I, H, L, O = (int(v) for v in g["dims"])
    w = golden_weights(g, L)
    f = lambda a: torch.from_numpy(a).to(device=cuda_device, dtype=torch.float16)
    conv_in = [[f(a) for a in w[0]], [f(a) for a in w[1]], [f(a) for a in w[2]], [f(a) for a in w[3]], f(w[4]), f(w[5])]
    out, _, _ = plstm.lstm_linear_forward(f(g["x"]), *conv_in, out_mode="last", check=True)
    assert_close16(out, g["regressor_out"], "regressor")
    seq, _, _ = plstm.lstm_linear_forward(f(g["x"]), *conv_in, out_mode="seq", check=True)
    assert_close16(seq[:, -1], g["regressor_out"], "seq last step")


def test_converted_regressor_module(cuda_device):
    m = plstm.StandardLSTMRegressor(5, 128, 24, 4).eval()
    native = m.to(cuda_device).half()
    conv = plstm.convert_regressor_module(native)
    assert "tc" in conv.backend_name
    x = _rand_x(64, 50, 5, torch.float16, cuda_device)
    with torch.inference_mode():
        ref = native(x)
    got = conv(x)
    assert got.shape == (64, 24)
    assert_close16(got, ref.double().cpu().numpy(), "vs native nn.LSTM (cuDNN)")
    seq, (h_n, c_n) = conv.forward_sequence(x)
    assert seq.shape == (64, 50, 24) and h_n.shape == (4, 64, 128)
    torch.testing.assert_close(seq[:, -1], got, rtol=0, atol=0)
    lstm = plstm.convert_lstm_module(native.lstm)
    hs, (h2, c2) = lstm(x)
    with torch.inference_mode():
        rh, (rh_n, rc_n) = native.lstm(x)
    assert_close16(hs, rh.double().cpu().numpy(), "PersistentLSTM out")
    assert_close16(h2, rh_n.double().cpu().numpy(), "PersistentLSTM h_n")


def test_repeat_first_row(cuda_device):
    src = torch.randn(3, 24, device=cuda_device).half()
    out = ext.repeat_first_row(src, 7)
    assert torch.equal(out, src[:1].expand(7, 24))


# ---------------------------------------------------------------------------------------
@pytest.mark.parametrize("mode", ["last", "seq"])
def test_tc_full_size_cfg2_sampled(cuda_device, mode):
    """Config 2 at full size (B=512, T=1000, f16); the oracle checks 24 sampled rows."""
    B, T, I, H, L, O = 512, 1000, 5, 128, 4, 24
    m = make_model(I, H, L, O, seed=0)
    w = weights_of(m, L, torch.float16, cuda_device)
    x = _rand_x(B, T, I, torch.float16, cuda_device)
    pw = core.PackedWeights(*w, out_mode=mode)
    assert pw.backend == "tc"
    out, h_n, c_n = pw.forward(x, check=True)
    rows = np.linspace(0, B - 1, 24).astype(int)
    r_out, r_h, r_c = oracle_of(x, *w, out_mode=mode, rows=rows)
    assert_close16(out[rows], r_out, "out")
    assert_close16(h_n[:, rows], r_h, "h_n")
    assert torch.isfinite(out.float()).all()


def test_tc_full_size_cfg5_varlen_sampled(cuda_device):
    """Config 5 shard on one GPU (B=512 of the 4096, lengths in [200, 1000])."""
    B, T, I, H, L, O = 512, 1000, 5, 128, 4, 24
    m = make_model(I, H, L, O, seed=0)
    w = weights_of(m, L, torch.float16, cuda_device)
    x = _rand_x(B, T, I, torch.float16, cuda_device)
    g = torch.Generator().manual_seed(2)
    lens = torch.randint(200, T + 1, (B,), generator=g, dtype=torch.int32)
    pw = core.PackedWeights(*w, out_mode="seq")
    out, h_n, c_n = pw.forward(x, lengths=lens.to(cuda_device), check=True)
    rows = np.linspace(0, B - 1, 16).astype(int)
    r_out, r_h, _ = oracle_of(x, *w, lengths=lens, out_mode="seq", rows=rows)
    assert_close16(out[rows], r_out, "out")
    assert_close16(h_n[:, rows], r_h, "h_n")


@pytest.mark.parametrize("spread", [True, False])
@pytest.mark.parametrize("B, mode", [(512, "seq"), (520, "last"), (700, "hseq")])
def test_tc_varlen_tile_height_choice(cuda_device, monkeypatch, spread, B, mode):
    """Variable-length batches past one wave of 32-row tiles enqueue both tile heights and
    pick one on the device.  A row's arithmetic does not depend on the other rows of its
    tile, so the result equals, bit for bit, both forced heights; sampled rows against the
    oracle.  Spread lengths favour 32-row tiles, equal lengths 64-row ones."""
    T, I, H, L, O = 120, 5, 128, 4, 24
    m = make_model(I, H, L, O, seed=40)
    w = weights_of(m, L, torch.float16, cuda_device)
    x = _rand_x(B, T, I, torch.float16, cuda_device, seed=41)
    g = torch.Generator().manual_seed(42)
    lens = torch.randint(1, T + 1, (B,), generator=g, dtype=torch.int32) if spread else \
        torch.full((B,), T, dtype=torch.int32)
    h0 = (0.3 * torch.randn(L, B, H, generator=g)).half().to(cuda_device)
    c0 = (0.3 * torch.randn(L, B, H, generator=g)).half().to(cuda_device)
    pw = core.PackedWeights(*w, out_mode=mode)
    assert pw.backend == "tc"
    run = lambda: pw.forward(x, lengths=lens.to(cuda_device), hx=(h0, c0), check=True)
    auto = run()
    for nt in ("32", "64"):
        monkeypatch.setenv("PLSTM_TC_NTILE", nt)
        forced = run()
        for a, f in zip(auto, forced):
            assert torch.equal(a, f), nt
    monkeypatch.delenv("PLSTM_TC_NTILE")
    rows = np.linspace(0, B - 1, 12).astype(int)
    r_out, r_h, r_c = oracle_of(x, *w, lengths=lens, hx=(h0, c0), out_mode=mode, rows=rows)
    assert_close16(auto[0][rows], r_out, "out")
    assert_close16(auto[1][:, rows], r_h, "h_n")
    assert_close16(auto[2][:, rows], r_c, "c_n")


def test_timeout_is_reported_not_hung(cuda_device):
    """A producer CTA that skips one h hand-off makes its consumer's bounded
    wait run out; the call returns PLSTM_ETIMEOUT and the context stays usable."""
    B, T, I, H, L, O = 32, 16, 5, 128, 4, 24
    m = make_model(I, H, L, O, seed=11)
    w = weights_of(m, L, torch.float16, cuda_device)
    x = _rand_x(B, T, I, torch.float16, cuda_device)
    pw = core.PackedWeights(*w, out_mode="last", backend="tc")
    with pytest.raises(plstm.PlstmError) as ei:
        pw.forward(x, check=True, timeout_ms=50, extra_flags=_lib.FLAG_TEST_DROP)
    assert ei.value.code == _lib.ETIMEOUT
    out, _, _ = pw.forward(x, check=True)
    r_out, _, _ = oracle_of(x, *w, out_mode="last")
    assert_close16(out, r_out, "after timeout")


@pytest.mark.parametrize("variant", [0, 15])
@pytest.mark.parametrize("rows", [16, 32])
def test_step_latency_probe(cuda_device, rows, variant):
    """The dependent-step probe finishes, reports its phases, and its step time is plausible:
    at least the sum of its own phases' MMA issue and no longer than a full wavefront step."""
    from persistent_lstm_hip_b200 import microbench

    r = microbench.step_latency(rows=rows, steps=4000, variant=variant)
    ph = r["phase_cycles"]
    assert 300 < r["cycles_per_step"] < 20000, r
    assert abs(sum(ph.values()) - r["cycles_per_step"]) < 0.05 * r["cycles_per_step"], r
    assert 0.1 < r["us_per_step"] < 10, r
    lib = _lib.load()
    out = torch.zeros(16, dtype=torch.int64, device=cuda_device)
    assert lib.plstm_diag_step_latency(24, 100, 0, out.data_ptr(), 0, None) == _lib.EINVAL


def test_unchecked_timeout_raises_by_the_next_call(cuda_device):
    """Without a synchronising check the failure of a forward is not lost: its status word
    is copied back asynchronously and the next forward on the device raises PLSTM_ETIMEOUT
    (the wait is host-armed: a producer skips one hand-off, bounded to 50 ms)."""
    B, T, I, H, L, O = 32, 16, 5, 128, 4, 24
    m = make_model(I, H, L, O, seed=11)
    w = weights_of(m, L, torch.float16, cuda_device)
    x = _rand_x(B, T, I, torch.float16, cuda_device)
    pw = core.PackedWeights(*w, out_mode="last", backend="tc")
    core.check_device_status(cuda_device)  # nothing pending from earlier tests
    pw.forward(x, check=False, timeout_ms=50, extra_flags=_lib.FLAG_TEST_DROP)  # returns without an error
    torch.cuda.synchronize()
    with pytest.raises(plstm.PlstmError) as ei:
        pw.forward(x, check=False)
    assert ei.value.code == _lib.ETIMEOUT
    assert "earlier forward" in str(ei.value)
    # Reported once; the context stays usable and later forwards are correct.
    out, _, _ = pw.forward(x, check=False)
    core.check_device_status(cuda_device)
    r_out, _, _ = oracle_of(x, *w, out_mode="last")
    assert_close16(out, r_out, "after timeout")
    # check_device_status waits for the copy itself.
    pw.forward(x, check=False, timeout_ms=50, extra_flags=_lib.FLAG_TEST_DROP)
    with pytest.raises(plstm.PlstmError):
        core.check_device_status(cuda_device)


@pytest.mark.parametrize("mode", ["seq", "last", "hseq"])
@pytest.mark.parametrize("varlen", [False, True])
def test_single_slot_wavefront_kernel(cuda_device, monkeypatch, mode, varlen):
    """The single-slot wavefront kernel (PLSTM_TC_KERNEL=1) stays selectable and exact."""
    monkeypatch.setenv("PLSTM_TC_KERNEL", "1")
    B, T, I, H, L, O = 50, 21, 5, 128, 3, 24
    m = make_model(I, H, L, O, seed=13)
    w = weights_of(m, L, torch.float16, cuda_device)
    x = _rand_x(B, T, I, torch.float16, cuda_device, seed=3)
    lens = _rand_lengths(B, T, lo=1) if varlen else None
    pw = core.PackedWeights(*w, out_mode=mode, backend="tc")
    out, h_n, c_n = pw.forward(x, lengths=None if lens is None else lens.to(cuda_device), check=True)
    r_out, r_h, r_c = oracle_of(x, *w, lengths=lens, out_mode=mode)
    assert_close16(out, r_out, "out")
    assert_close16(h_n, r_h, "h_n")
    assert_close16(c_n, r_c, "c_n")


# ---------------------------------------------------------------------------------------
# Generic shapes on the H = 128 tensor-core kernel: layer-0 inputs wider than one
# 16-column MMA step (I <= 128) and stacks of up to 8 layers (16-CTA clusters).
@pytest.mark.parametrize("I", [16, 17, 40, 128])
@pytest.mark.parametrize("mode", ["seq", "last"])
def test_tc_wide_input(cuda_device, I, mode):
    B, T, H, L, O = 70, 19, 128, 3, 24
    m = make_model(I, H, L, O, seed=20 + I)
    w = weights_of(m, L, torch.float16, cuda_device)
    x = _rand_x(B, T, I, torch.float16, cuda_device, seed=I)
    pw = core.PackedWeights(*w, out_mode=mode, backend="tc")
    assert pw.backend == "tc"
    out, h_n, c_n = pw.forward(x, check=True)
    r_out, r_h, r_c = oracle_of(x, *w, out_mode=mode)
    assert_close16(out, r_out, "out")
    assert_close16(h_n, r_h, "h_n")
    assert_close16(c_n, r_c, "c_n")


@pytest.mark.parametrize("L", [5, 6, 8])
def test_tc_more_layers(cuda_device, L):
    B, T, I, H, O = 40, 17, 5, 128, 24
    m = make_model(I, H, L, O, seed=30 + L)
    w = weights_of(m, L, torch.float16, cuda_device)
    x = _rand_x(B, T, I, torch.float16, cuda_device, seed=L)
    pw = core.PackedWeights(*w, out_mode="seq", backend="tc")
    assert pw.backend == "tc"
    out, h_n, c_n = pw.forward(x, check=True)
    r_out, r_h, r_c = oracle_of(x, *w, out_mode="seq")
    assert_close16(out, r_out, "out")
    assert_close16(h_n, r_h, "h_n")
    assert_close16(c_n, r_c, "c_n")


@pytest.mark.parametrize("mode", ["seq", "hseq"])
def test_tc_wide_input_deep_varlen_state_bf16(cuda_device, mode):
    B, T, I, H, L, O = 77, 23, 64, 128, 6, 12
    m = make_model(I, H, L, O, seed=41)
    w = weights_of(m, L, torch.bfloat16, cuda_device)
    x = _rand_x(B, T, I, torch.bfloat16, cuda_device, seed=5)
    lens = _rand_lengths(B, T, lo=0)
    g = torch.Generator().manual_seed(8)
    hx = ((0.5 * torch.randn(L, B, H, generator=g)).to(cuda_device, torch.bfloat16),
          (0.5 * torch.randn(L, B, H, generator=g)).to(cuda_device, torch.bfloat16))
    pw = core.PackedWeights(*w, out_mode=mode, backend="tc")
    out, h_n, c_n = pw.forward(x, lengths=lens.to(cuda_device), hx=hx, check=True)
    r_out, r_h, r_c = oracle_of(x, *w, lengths=lens, hx=hx, out_mode=mode)
    assert_close16(out, r_out, "out")
    assert_close16(h_n, r_h, "h_n")
    assert_close16(c_n, r_c, "c_n")


def test_tc_wide_input_ignores_single_slot_request(cuda_device, monkeypatch):
    """PLSTM_TC_KERNEL=1 selects the single-slot kernel only for inputs of <= 16 columns."""
    monkeypatch.setenv("PLSTM_TC_KERNEL", "1")
    B, T, I, H, L, O = 30, 11, 33, 128, 2, 24
    m = make_model(I, H, L, O, seed=43)
    w = weights_of(m, L, torch.float16, cuda_device)
    x = _rand_x(B, T, I, torch.float16, cuda_device, seed=6)
    pw = core.PackedWeights(*w, out_mode="last", backend="tc")
    out, h_n, c_n = pw.forward(x, check=True)
    r_out, r_h, r_c = oracle_of(x, *w, out_mode="last")
    assert_close16(out, r_out, "out")
    assert_close16(h_n, r_h, "h_n")


def test_tc_rejects_beyond_envelope(cuda_device):
    """Shapes past both tensor-core envelopes (H = 128 wavefront: I <= 128, L <= 8; layer
    path: I <= 128, L <= 16) are refused by the forced TC backend and served by the generic
    kernel under "auto"; H = 128 with 9 layers runs on the layer path."""
    assert core.select_backend(input_size=40, hidden_size=128, num_layers=9, output_size=24,
                               dtype=torch.float16, device=cuda_device.index or 0) == "tc"
    for I, L in [(129, 2), (5, 17)]:
        assert core.select_backend(input_size=I, hidden_size=128, num_layers=L, output_size=24,
                                   dtype=torch.float16, device=cuda_device.index or 0) == "simt"
        with pytest.raises(_lib.PlstmError):
            core.select_backend(input_size=I, hidden_size=128, num_layers=L, output_size=24,
                                dtype=torch.float16, backend="tc", device=cuda_device.index or 0)


# Hidden sizes below 128 run on the H = 128 wavefront kernel with the extra units zero
# padded (zero weights, bias and state: they stay zero and feed nothing).
@pytest.mark.parametrize("H", [1, 40, 64, 100])
@pytest.mark.parametrize("mode", ["seq", "last", "hseq"])
def test_tc_small_hidden_sizes_padded(cuda_device, H, mode):
    B, T, I, L, O = 37, 13, 5, 3, 24
    m = make_model(I, H, L, O, seed=50 + H)
    w = weights_of(m, L, torch.float16, cuda_device)
    x = _rand_x(B, T, I, torch.float16, cuda_device, seed=H)
    pw = core.PackedWeights(*w, out_mode=mode)
    assert pw.backend == "tc"
    out, h_n, c_n = pw.forward(x, check=True)
    r_out, r_h, r_c = oracle_of(x, *w, out_mode=mode)
    assert_close16(out, r_out, "out")
    assert_close16(h_n, r_h, "h_n")
    assert_close16(c_n, r_c, "c_n")


def test_tc_small_hidden_varlen_state_bf16(cuda_device):
    B, T, I, H, L, O = 51, 19, 20, 72, 4, 10
    m = make_model(I, H, L, O, seed=61)
    w = weights_of(m, L, torch.bfloat16, cuda_device)
    x = _rand_x(B, T, I, torch.bfloat16, cuda_device, seed=9)
    lens = _rand_lengths(B, T, lo=0)
    g = torch.Generator().manual_seed(10)
    hx = ((0.5 * torch.randn(L, B, H, generator=g)).to(cuda_device, torch.bfloat16),
          (0.5 * torch.randn(L, B, H, generator=g)).to(cuda_device, torch.bfloat16))
    for mode in ("seq", "hseq"):
        pw = core.PackedWeights(*w, out_mode=mode, backend="tc")
        out, h_n, c_n = pw.forward(x, lengths=lens.to(cuda_device), hx=hx, check=True, c_n_f32=True)
        r_out, r_h, r_c = oracle_of(x, *w, lengths=lens, hx=hx, out_mode=mode)
        assert_close16(out, r_out, "out")
        assert_close16(h_n, r_h, "h_n")
        assert_close16(c_n, r_c, "c_n")


def test_every_output_element_written(cuda_device):
    """[B,T,O], [B,O] and [B,T,H] outputs land in a buffer pre-filled with NaN: every element must
    be written (zeros past each row's length included), also for a tile slot whose rows all have
    length 0 and for output widths whose rows are stored in 16-, 8-, 4- and 2-byte pieces."""
    lib = _lib.load()
    for (B, T, H, L, O, ntile) in [(40, 9, 128, 2, 24, "32"), (70, 7, 128, 3, 12, "64"), (50, 6, 128, 2, 10, None),
                                   (33, 5, 96, 2, 7, "64"), (45, 5, 96, 2, 5, "32"), (200, 5, 128, 2, 24, "48")]:
        m = make_model(5, H, L, O, seed=B)
        w = weights_of(m, L, torch.float16, cuda_device)
        x = _rand_x(B, T, 5, torch.float16, cuda_device, seed=B + 1)
        lens = _rand_lengths(B, T, seed=B + 2, lo=0)
        lens[B - 20:] = 0  # the last rows (a whole 16-row slot) have length 0
        varlen = ntile != "48"  # 48-row tiles take uniform lengths only
        os.environ.pop("PLSTM_TC_NTILE", None)
        if ntile:
            os.environ["PLSTM_TC_NTILE"] = ntile
        try:
            for mode, shape in (("seq", (B, T, O)), ("last", (B, O)), ("hseq", (B, T, H))):
                pw = core.PackedWeights(*w, out_mode=mode, backend="tc")
                d = pw.desc(batch=B, seq_len=T, extra_flags=_lib.FLAG_SYNC_CHECK)
                nb = ctypes.c_size_t(0)
                _lib.check(lib.plstm_workspace_size(ctypes.byref(d), ctypes.byref(nb)))
                ws = torch.zeros(max(int(nb.value), 256), dtype=torch.uint8, device=cuda_device)
                out = torch.full(shape, float("nan"), dtype=torch.float16, device=cuda_device)
                ld = lens.to(cuda_device) if varlen else None
                _lib.check(lib.plstm_forward_packed(ctypes.byref(d), pw.blob.data_ptr(), x.data_ptr(),
                                                    ld.data_ptr() if ld is not None else None, None, None,
                                                    out.data_ptr(), None, None, ws.data_ptr(), ws.numel(),
                                                    torch.cuda.current_stream().cuda_stream))
                torch.cuda.synchronize()
                assert not torch.isnan(out).any(), f"{mode} B={B} O={O} ntile={ntile}: unwritten elements"
                r_out, _, _ = oracle_of(x, *w, lengths=lens if varlen else None, out_mode=mode)
                assert_close16(out, r_out, f"{mode} B={B} O={O}")
        finally:
            os.environ.pop("PLSTM_TC_NTILE", None)
