"""Drop-in for functions of the reference's `miopen_adaptive_lstm_hip._C` extension.

Mirrors miopen_adaptive_lstm_hip/csrc/bindings.cpp:5-78 function by function
as thin torch-tensor shims over the C ABI (include/plstm.h).
"""
from __future__ import annotations

import ctypes

import torch

from . import _lib
from .core import _stream, device_status

_DT = {torch.float16: _lib.F16, torch.bfloat16: _lib.BF16}


def adaptive_lstm_input_gemm_forward_workspace(input_2d: torch.Tensor, weight_ih_t: torch.Tensor,
                                               gate: torch.Tensor) -> torch.Tensor:
    """gate[N_rows, 4H] = input_2d[N_rows, K] @ weight_ih_t[K, 4H] (no bias), into the caller's
    `gate` workspace; returns `gate` (bindings.cpp:38-41, adaptive_lstm_hip.cu:2355-2385).
    f16 (as the reference) or bf16, f32 accumulation, tcgen05 tensor cores."""
    if not (input_2d.is_cuda and weight_ih_t.is_cuda and gate.is_cuda):
        raise ValueError("adaptive input projection GEMM expects CUDA tensors")
    if not (input_2d.dtype == weight_ih_t.dtype == gate.dtype and input_2d.dtype in _DT):
        raise ValueError("adaptive input projection GEMM expects FP16 (or BF16) tensors of one dtype")
    if not (input_2d.dim() == 2 and weight_ih_t.dim() == 2 and gate.dim() == 2):
        raise ValueError("expected input [N,K], weight_ih_t [K,4H], gate [N,4H]")
    x = input_2d.contiguous()
    w = weight_ih_t.contiguous()
    if x.size(1) != w.size(0) or gate.size(0) != x.size(0) or gate.size(1) != w.size(1) or not gate.is_contiguous():
        raise ValueError("adaptive input projection GEMM received incompatible shapes")
    lib = _lib.load()
    with torch.cuda.device(gate.device):
        _lib.check(lib.plstm_input_gemm(x.data_ptr(), int(x.size(0)), int(x.size(1)), w.data_ptr(), int(w.size(1)),
                                        _DT[x.dtype], gate.data_ptr(), _stream(gate.device)))
    return gate


# ---- hidden updates -------------------------------------------------------------------
# Every hidden-update function of the reference extension (bindings.cpp:6-36, 42-78;
# adaptive_lstm_hip.h:5-170) runs the same recurrence over a precomputed input
# projection, from h = c = 0:  gates = gate_proj[:, t] + bias + W_hh h_{t-1}.  They differ
# in the gate / weight layouts they take and in which tensors they fill; here each is a
# shim over plstm_hidden_update (tensor cores for H in {128, 256, 512}, FFMA otherwise).
# The reference's tuning knobs (read_block, items_per_group, partitions, fast_act,
# recurrent_compute) select among its own HIP kernels and have no effect here.

_W_NATIVE, _W_TRANSPOSED, _W_MMAC = _lib.W_NATIVE, _lib.W_TRANSPOSED, _lib.W_MMAC


def _hidden_update(what, gate, weight, w_layout, bias, h_state, c_state, out, write_sequence, seq_major=False):
    lib = _lib.load()
    dt = gate.dtype
    codes = dict(_DT)
    codes[torch.float32] = _lib.F32  # the C entry point also serves f32 (FFMA kernel)
    if dt not in codes:
        raise ValueError(f"{what} expects FP16, BF16 or FP32 data")
    if seq_major:
        T, B, G = (int(v) for v in gate.shape)
    else:
        B, T, G = (int(v) for v in gate.shape)
    H = G // 4
    flags = (_lib.HU_SEQ_MAJOR if seq_major else 0) | (_lib.HU_WRITE_SEQUENCE if write_sequence else 0)
    dev = gate.device
    nbytes = ctypes.c_size_t(0)
    _lib.check(lib.plstm_hidden_update_workspace_size(B, T, H, codes[dt], flags, dev.index or 0, ctypes.byref(nbytes)))
    ws = torch.empty(max(int(nbytes.value), 1), dtype=torch.uint8, device=dev)
    g = gate.contiguous()
    w = weight.contiguous()
    b = None if bias is None else bias.contiguous()
    watcher = device_status(dev)
    watcher.poll()  # a device failure of an earlier call surfaces here
    with torch.cuda.device(dev):
        _lib.check(lib.plstm_hidden_update(g.data_ptr(), B, T, H, w.data_ptr(), w_layout,
                                           None if b is None else b.data_ptr(), codes[dt], flags, h_state.data_ptr(),
                                           c_state.data_ptr(), out.data_ptr(), ws.data_ptr(), ws.numel(),
                                           _stream(dev)))
    watcher.watch(ws, torch.cuda.current_stream(dev))


def _check_cuda(what, *ts):
    if not all(t.is_cuda for t in ts):
        raise ValueError(f"{what} expects CUDA tensors")


def _check_types(what, gate, weight, bias, h_state=None, c_state=None, out=None):
    dt = gate.dtype
    ok = dt in _DT and weight.dtype == dt and (bias is None or bias.dtype == dt)
    ok = ok and all(t is None or t.dtype == dt for t in (h_state, out))
    ok = ok and (c_state is None or c_state.dtype == torch.float32)
    if not ok:
        raise ValueError(f"{what} expects FP16 (or BF16) data and FP32 cell state")


def _weight_layout(what, weight, H):
    if weight.dim() == 2 and tuple(weight.shape) == (4 * H, H):
        return _W_NATIVE
    if weight.dim() == 2 and tuple(weight.shape) == (H, 4 * H):
        return _W_TRANSPOSED
    raise ValueError(f"{what}: weight_hh must be [4H, H] or [H, 4H]")


def _new_outputs(gate, write_sequence, seq_major=False):
    if seq_major:
        T, B, G = gate.shape
    else:
        B, T, G = gate.shape
    H = G // 4
    h = torch.empty(B, H, dtype=gate.dtype, device=gate.device)
    c = torch.empty(B, H, dtype=torch.float32, device=gate.device)
    if write_sequence:
        out = torch.empty((T, B, H) if seq_major else (B, T, H), dtype=gate.dtype, device=gate.device)
    else:
        out = torch.empty(B, H, dtype=gate.dtype, device=gate.device)
    return h, c, out


def _allocating(what, gate_proj, weight_hh, bias, write_sequence, hidden=None):
    """Shared body of the reference's allocating variants: gate [B,T,4H], weight_hh [4H,H],
    bias [4H]; returns a new [B,T,H] (write_sequence) or [B,H] tensor."""
    _check_cuda(what, gate_proj, weight_hh, bias)
    _check_types(what, gate_proj, weight_hh, bias)
    if not (gate_proj.dim() == 3 and weight_hh.dim() == 2 and bias.dim() == 1):
        raise ValueError("expected gate [B,T,4H], weight_hh [4H,H], bias [4H]")
    G = int(gate_proj.shape[2])
    H = G // 4
    if G != 4 * H or tuple(weight_hh.shape) != (4 * H, H) or int(bias.shape[0]) != G or (hidden and H != hidden):
        raise ValueError(f"incompatible {what} shapes")
    h, c, out = _new_outputs(gate_proj, write_sequence)
    _hidden_update(what, gate_proj, weight_hh, _W_NATIVE, bias, h, c, out, write_sequence)
    return out


def adaptive_lstm_hidden_update_forward(gate_proj, weight_hh, bias, write_sequence, read_block, items_per_group):
    """Hidden update over gate_proj [B,T,4H] (adaptive_lstm_hip.cu:1497-1545)."""
    return _allocating("adaptive hidden update", gate_proj, weight_hh, bias, write_sequence)


def adaptive_lstm_hidden_update_partitioned_forward(gate_proj, weight_hh, bias, write_sequence, partitions):
    """Partitioned hidden update (the partitioning is a HIP launch detail)."""
    if int(partitions) < 1:
        raise ValueError("partitions must be >= 1")
    return _allocating("adaptive partitioned hidden update", gate_proj, weight_hh, bias, write_sequence)


def adaptive_lstm_h128_cached_update_forward(gate_proj, weight_hh, bias, write_sequence):
    return _allocating("adaptive H128 cached update", gate_proj, weight_hh, bias, write_sequence, hidden=128)


def adaptive_lstm_h128_cached_b4_update_forward(gate_proj, weight_hh, bias, write_sequence):
    return _allocating("adaptive H128 cached B4 update", gate_proj, weight_hh, bias, write_sequence, hidden=128)


def adaptive_lstm_h128_cached_b8_update_forward(gate_proj, weight_hh, bias, write_sequence):
    return _allocating("adaptive H128 cached B8 update", gate_proj, weight_hh, bias, write_sequence, hidden=128)


def adaptive_lstm_h128_gemm_scan_update_forward(gate_proj, weight_hh, bias, write_sequence, read_block):
    return _allocating("adaptive H128 GEMM scan", gate_proj, weight_hh, bias, write_sequence, hidden=128)


def _workspace_variant(what, gate_proj, weight_hh, bias, h_state, c_state, out, write_sequence, hidden=None,
                       w_layout=None):
    """Shared body of the workspace variants: fills h_state [B,H], c_state [B,H] (f32) and out
    ([B,T,H] or [B,H]); returns out (write_sequence) or h_state, as the reference does."""
    _check_cuda(what, gate_proj, weight_hh, bias, h_state, c_state, out)
    _check_types(what, gate_proj, weight_hh, bias, h_state, c_state, out)
    if not (gate_proj.dim() == 3 and bias.dim() == 1 and h_state.dim() == 2 and c_state.dim() == 2):
        raise ValueError("expected gate [B,T,4H], weight_hh [H,4H] or [4H,H], state [B,H]")
    B, T, G = (int(v) for v in gate_proj.shape)
    H = G // 4
    if G != 4 * H or (hidden and H != hidden):
        raise ValueError(f"{what} received incompatible shapes")
    layout = w_layout if w_layout is not None else _weight_layout(what, weight_hh, H)
    out_ok = (tuple(out.shape) == (B, T, H)) if write_sequence else (tuple(out.shape) == (B, H))
    if (int(bias.shape[0]) != G or tuple(h_state.shape) != (B, H) or tuple(c_state.shape) != (B, H)
            or not out_ok):
        raise ValueError(f"{what} received incompatible shapes")
    if not (h_state.is_contiguous() and c_state.is_contiguous() and out.is_contiguous()):
        raise ValueError(f"{what} workspace tensors must be contiguous")
    _hidden_update(what, gate_proj, weight_hh, layout, bias, h_state, c_state, out, write_sequence)
    return out if write_sequence else h_state


def adaptive_lstm_h128_gemm_scan_update_forward_workspace(gate_proj, weight_hh, bias, h_state, c_state, recur, out,
                                                          write_sequence, read_block):
    return _workspace_variant("adaptive H128 GEMM scan workspace", gate_proj, weight_hh, bias, h_state, c_state, out,
                              write_sequence, hidden=128)


def adaptive_lstm_h256_gemm_scan_update_forward_workspace(gate_proj, weight_hh, bias, h_state, c_state, recur, out,
                                                          write_sequence, read_block, recurrent_compute):
    return _workspace_variant("adaptive fixed GEMM scan workspace", gate_proj, weight_hh, bias, h_state, c_state, out,
                              write_sequence, hidden=256)


def adaptive_lstm_h512_gemm_scan_update_forward_workspace(gate_proj, weight_hh, bias, h_state, c_state, recur, out,
                                                          write_sequence, read_block, recurrent_compute):
    return _workspace_variant("adaptive fixed GEMM scan workspace", gate_proj, weight_hh, bias, h_state, c_state, out,
                              write_sequence, hidden=512)


def adaptive_lstm_h256_gate_accum_update_forward_workspace(gate_proj, weight_hh, bias, h_state, c_state, out,
                                                           write_sequence, read_block):
    return _workspace_variant("adaptive fixed gate accum workspace", gate_proj, weight_hh, bias, h_state, c_state, out,
                              write_sequence, hidden=256)


def adaptive_lstm_h512_gate_accum_update_forward_workspace(gate_proj, weight_hh, bias, h_state, c_state, out,
                                                           write_sequence, read_block):
    return _workspace_variant("adaptive fixed gate accum workspace", gate_proj, weight_hh, bias, h_state, c_state, out,
                              write_sequence, hidden=512)


def adaptive_lstm_h128_persistent_mmac_update_forward_workspace(gate_proj, weight_hh, bias, h_state, c_state, out,
                                                                write_sequence, read_block, fast_act):
    return _workspace_variant("adaptive H128 persistent update", gate_proj, weight_hh, bias, h_state, c_state, out,
                              write_sequence, hidden=128)


def adaptive_lstm_gemm_scan_update_forward_workspace(gate_proj, weight_hh, bias, h_state, c_state, recur, out,
                                                     write_sequence, read_block):
    """Any hidden size (FFMA kernel unless H is 128, 256 or 512)."""
    return _workspace_variant("adaptive generic GEMM scan workspace", gate_proj, weight_hh, bias, h_state, c_state,
                              out, write_sequence)


def adaptive_lstm_h128_seqmajor_accum_update_forward(gate_seq, weight_hh, h_state, c_state, seq_out, write_sequence,
                                                     read_block):
    """Seq-major variant: gate_seq [T,B,512] already holds the bias; seq_out [T,B,128] or [B,128].
    Unlike the reference (which accumulates W_hh h into gate_seq in place), gate_seq is not modified."""
    what = "adaptive H128 seqmajor accum"
    _check_cuda(what, gate_seq, weight_hh, h_state, c_state, seq_out)
    _check_types(what, gate_seq, weight_hh, None, h_state, c_state, seq_out)
    if not (gate_seq.dim() == 3 and weight_hh.dim() == 2 and h_state.dim() == 2 and c_state.dim() == 2):
        raise ValueError("expected gate [T,B,512], weight_hh [128,512] or [512,128], state [B,128]")
    T, B, G = (int(v) for v in gate_seq.shape)
    out_ok = (tuple(seq_out.shape) == (T, B, 128)) if write_sequence else (tuple(seq_out.shape) == (B, 128))
    if G != 512 or tuple(h_state.shape) != (B, 128) or tuple(c_state.shape) != (B, 128) or not out_ok:
        raise ValueError(f"{what} received incompatible shapes")
    layout = _weight_layout(what, weight_hh, 128)
    _hidden_update(what, gate_seq, weight_hh, layout, None, h_state, c_state, seq_out, write_sequence, seq_major=True)
    return seq_out if write_sequence else h_state


def _mmac_packed(H, gate_proj, packed_weight, bias, h_state, c_state, out, profile_out, write_sequence, read_block,
                 variant):
    """MMAC-packed weight (`_pack_mmac_weight` layout, H*H*4 values).  variant 3 is the full
    update; variants 0-2 are profiling cut-downs of the reference's AMD MMAC kernel (partial
    gate math written to profile_out) with no counterpart here."""
    what = "adaptive packed MMAC kernel"
    if int(variant) != 3:
        raise ValueError(f"{what}: only variant 3 (the full update) is provided; variants 0-2 are AMD MMAC "
                         "profiling cut-downs")
    if packed_weight.dim() != 1 or int(packed_weight.numel()) != H * H * 4:
        raise ValueError(f"{what} received incompatible shapes")
    _check_cuda(what, profile_out)
    return _workspace_variant(what, gate_proj, packed_weight, bias, h_state, c_state, out, write_sequence, hidden=H,
                              w_layout=_W_MMAC)


def adaptive_lstm_h128_mmac_packed_variant_forward_workspace(gate_proj, packed_weight, bias, h_state, c_state, out,
                                                             profile_out, write_sequence, read_block, variant):
    return _mmac_packed(128, gate_proj, packed_weight, bias, h_state, c_state, out, profile_out, write_sequence,
                        read_block, variant)


def adaptive_lstm_h256_mmac_packed_variant_forward_workspace(gate_proj, packed_weight, bias, h_state, c_state, out,
                                                             profile_out, write_sequence, read_block, variant):
    return _mmac_packed(256, gate_proj, packed_weight, bias, h_state, c_state, out, profile_out, write_sequence,
                        read_block, variant)


def adaptive_lstm_h512_mmac_packed_variant_forward_workspace(gate_proj, packed_weight, bias, h_state, c_state, out,
                                                             profile_out, write_sequence, read_block, variant):
    return _mmac_packed(512, gate_proj, packed_weight, bias, h_state, c_state, out, profile_out, write_sequence,
                        read_block, variant)
