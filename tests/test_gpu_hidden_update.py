"""GPU parity of plstm_hidden_update (the recurrence over precomputed input
projections behind every hidden-update function of the reference's adaptive
extension) and of the `_C` shims.  The checker is the pinned oracle, run as a
one-layer LSTM whose input is the projection itself (W_ih = identity, input size
4H), on the same 16-bit-rounded values the device saw."""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from helpers import assert_close16, oracle_of
from test_hidden_update_cpu import mmac_index
import persistent_lstm_hip_b200 as plstm
from persistent_lstm_hip_b200 import _lib, adaptive_ext as C

pytestmark = pytest.mark.gpu


def _case(B, T, H, dtype, dev, seed=0):
    g = torch.Generator().manual_seed(seed)
    s = 1.0 / np.sqrt(H)
    gp = (torch.randn(B, T, 4 * H, generator=g) * 0.8).to(dev, dtype)
    w = ((torch.rand(4 * H, H, generator=g) * 2 - 1) * s).to(dev, dtype)
    b = ((torch.rand(4 * H, generator=g) * 2 - 1) * s).to(dev, dtype)
    return gp, w, b


def _oracle(gp, w, b, seq_major=False):
    """(out [B,T,H], h [B,H], c [B,H]) from the oracle: one layer, input = gate_proj, W_ih = I."""
    x = gp.transpose(0, 1) if seq_major else gp
    G = x.shape[2]
    eye = torch.eye(G, dtype=x.dtype, device=x.device)
    out, h_n, c_n = oracle_of(x, [eye], [w], [b], [torch.zeros_like(b)], None, None, out_mode="hseq")
    return out, h_n[0], c_n[0]


def _mmac_pack(w):
    H = w.shape[1]
    wc = w.cpu()
    packed = torch.empty(4 * H * H, dtype=w.dtype)
    idx = torch.tensor([[mmac_index(H, r, k) for k in range(H)] for r in range(4 * H)])
    packed[idx.reshape(-1)] = wc.reshape(-1)
    return packed.to(w.device)


def _call(gp, w, layout, b, write_sequence, seq_major=False):
    if seq_major:
        T, B, G = gp.shape
    else:
        B, T, G = gp.shape
    H = G // 4
    h = torch.full((B, H), float("nan"), dtype=gp.dtype, device=gp.device)
    c = torch.full((B, H), float("nan"), dtype=torch.float32, device=gp.device)
    out = torch.full(((T, B, H) if seq_major else (B, T, H)) if write_sequence else (B, H), float("nan"),
                     dtype=gp.dtype, device=gp.device)
    C._hidden_update("test", gp, w, layout, b, h, c, out, write_sequence, seq_major=seq_major)
    torch.cuda.synchronize()
    return out, h, c


@pytest.mark.parametrize("H", [128, 256, 512, 64])
@pytest.mark.parametrize("write_sequence", [True, False])
def test_hidden_update_matches_oracle(cuda_device, H, write_sequence):
    B, T = 70, 9
    dtype = torch.bfloat16 if H == 512 else torch.float16
    gp, w, b = _case(B, T, H, dtype, cuda_device, seed=H)
    out, h, c = _call(gp, w, _lib.W_NATIVE, b, write_sequence)
    r_out, r_h, r_c = _oracle(gp, w, b)
    assert_close16(out, r_out if write_sequence else r_h, "out")
    assert_close16(h, r_h, "h_state")
    assert_close16(c, r_c, "c_state")


@pytest.mark.parametrize("layout", ["transposed", "mmac"])
def test_hidden_update_weight_layouts(cuda_device, layout):
    B, T, H = 33, 7, 128
    gp, w, b = _case(B, T, H, torch.float16, cuda_device, seed=3)
    wl = w.t().contiguous() if layout == "transposed" else _mmac_pack(w)
    code = _lib.W_TRANSPOSED if layout == "transposed" else _lib.W_MMAC
    out, h, c = _call(gp, wl, code, b, True)
    ref, _, _ = _call(gp, w, _lib.W_NATIVE, b, True)
    assert torch.equal(out, ref)


def test_hidden_update_seq_major_and_f32(cuda_device):
    B, T, H = 20, 6, 128
    gp, w, b = _case(B, T, H, torch.float16, cuda_device, seed=4)
    out, h, c = _call(gp.transpose(0, 1).contiguous(), w, _lib.W_NATIVE, b, True, seq_major=True)
    ref, rh, rc = _call(gp, w, _lib.W_NATIVE, b, True)
    assert torch.equal(out.transpose(0, 1), ref) and torch.equal(h, rh)
    # f32 runs the FFMA kernel; within the f32 tolerance of the oracle.
    g32, w32, b32 = gp.float(), w.float(), b.float()
    o32, h32, c32 = _call(g32, w32, _lib.W_NATIVE, b32, True)
    r_out, r_h, r_c = _oracle(g32, w32, b32)
    assert (o32.double().cpu() - torch.as_tensor(r_out)).abs().max().item() <= 1e-4


def test_adaptive_shims(cuda_device):
    """Every hidden-update function of the reference extension returns what the
    generic one computes, with the reference's return conventions."""
    B, T = 12, 5
    for H in (128, 256, 512):
        gp, w, b = _case(B, T, H, torch.float16, cuda_device, seed=H + 1)
        r_out, r_h, r_c = _oracle(gp, w, b)
        seq = C.adaptive_lstm_hidden_update_forward(gp, w, b, True, 4, 64)
        assert_close16(seq, r_out, f"H{H} hidden_update")
        last = C.adaptive_lstm_hidden_update_partitioned_forward(gp, w, b, False, 2)
        assert_close16(last, r_h, f"H{H} partitioned")
        h = torch.empty(B, H, dtype=gp.dtype, device=cuda_device)
        c = torch.empty(B, H, dtype=torch.float32, device=cuda_device)
        out = torch.empty(B, T, H, dtype=gp.dtype, device=cuda_device)
        recur = torch.empty(B, 4 * H, dtype=gp.dtype, device=cuda_device)
        got = C.adaptive_lstm_gemm_scan_update_forward_workspace(gp, w.t().contiguous(), b, h, c, recur, out, True, 1)
        assert got is out
        assert_close16(out, r_out, f"H{H} generic workspace")
        assert_close16(c, r_c, f"H{H} c_state")
        if H == 128:
            for fn in (C.adaptive_lstm_h128_cached_update_forward, C.adaptive_lstm_h128_cached_b4_update_forward,
                       C.adaptive_lstm_h128_cached_b8_update_forward):
                assert_close16(fn(gp, w, b, True), r_out, fn.__name__)
            assert_close16(C.adaptive_lstm_h128_gemm_scan_update_forward(gp, w, b, False, 2), r_h, "h128 gemm scan")
            hs = C.adaptive_lstm_h128_gemm_scan_update_forward_workspace(gp, w, b, h, c, recur, out[:, 0].contiguous(),
                                                                         False, 4)
            assert hs is h
            assert_close16(h, r_h, "h128 gemm scan workspace")
            assert_close16(C.adaptive_lstm_h128_persistent_mmac_update_forward_workspace(
                gp, w, b, h, c, out, True, 4, 1), r_out, "h128 persistent")
            # seq-major: the bias is folded into gate_seq by the caller.
            gs = (gp.float() + b.float()).to(gp.dtype).transpose(0, 1).contiguous()
            so = torch.empty(T, B, H, dtype=gp.dtype, device=cuda_device)
            C.adaptive_lstm_h128_seqmajor_accum_update_forward(gs, w, h, c, so, True, 1)
            r2, _, _ = _oracle(gs, w, torch.zeros_like(b), seq_major=True)
            assert_close16(so.transpose(0, 1), r2, "h128 seqmajor")
        else:
            fn_scan = getattr(C, f"adaptive_lstm_h{H}_gemm_scan_update_forward_workspace")
            fn_acc = getattr(C, f"adaptive_lstm_h{H}_gate_accum_update_forward_workspace")
            assert_close16(fn_scan(gp, w, b, h, c, recur, out, True, 1, 0), r_out, f"h{H} gemm scan")
            assert_close16(fn_acc(gp, w, b, h, c, out, True, 1), r_out, f"h{H} gate accum")
        packed = _mmac_pack(w)
        prof = torch.empty(B, 4 * H, dtype=gp.dtype, device=cuda_device)
        fn_p = getattr(C, f"adaptive_lstm_h{H}_mmac_packed_variant_forward_workspace")
        assert_close16(fn_p(gp, packed, b, h, c, out, prof, True, 1, 3), r_out, f"h{H} mmac packed")
        with pytest.raises(ValueError):
            fn_p(gp, packed, b, h, c, out, prof, True, 1, 0)


def test_adaptive_regressor_matches_persistent(cuda_device):
    from helpers import make_model
    from persistent_lstm_hip_b200 import adaptive

    m = make_model(5, 128, 2, 24, seed=8).to(cuda_device).half()
    x = torch.randn(10, 30, 5, generator=torch.Generator().manual_seed(2)).to(cuda_device, torch.float16)
    a = adaptive.convert_regressor_module(m)
    p = plstm.convert_regressor_module(m)
    assert torch.equal(a(x), p(x))
    with pytest.raises(RuntimeError):
        a.train()(x)
