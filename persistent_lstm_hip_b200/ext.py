"""Drop-in for the reference's pybind11 module `persistent_lstm_hip_ext`.

Same ten function names and argument order as
persistent_lstm_hip/csrc/bindings.cpp:154-165; each is a thin torch-tensor
shim over one C-ABI entry point of include/plstm.h.  Inputs are f16 CUDA
tensors as in the reference; the bias arguments are the pre-summed
b_ih + b_hh the reference's wrapper passes (model.py:552-561).  Shape errors
raise ValueError (the reference throws std::invalid_argument,
persistent_lstm_op.cpp:7-11).  CPU tensors raise: the reference silently ran
its ATen CPU loop there (persistent_lstm_op.cpp:55-70); this library has no
CPU path.
"""
from __future__ import annotations

import ctypes
from typing import Sequence

import torch

from . import _lib
from .core import _stream, device_status


def _check(cond: bool, msg: str) -> None:
    if not cond:
        raise ValueError(msg)


def _cuda_f16(t: torch.Tensor, name: str, device) -> torch.Tensor:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a tensor")
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (no CPU implementation)")
    if t.device != device:
        raise ValueError(f"{name} is on {t.device}, expected {device}")
    if t.dtype != torch.float16:
        raise ValueError(f"{name} must be float16")
    return t.contiguous()


def _ref4_call(fn_name: str, x, tensors, *, hidden_size: int, ih_kpair_k: int = 0):
    """Shared body of the fixed 4-layer entry points: 12 LSTM tensors + 2 head tensors."""
    _check(isinstance(x, torch.Tensor) and x.dim() == 3, "x must be [B, T, I]")
    _check(len(tensors) == 14, "expected 4 x (weight_ih, weight_hh, bias) + linear_weight, linear_bias")
    dev = x.device
    x = _cuda_f16(x, "x", dev)
    ts = [_cuda_f16(t, f"arg{i}", dev) for i, t in enumerate(tensors)]
    w_ih = [ts[3 * l] for l in range(4)]
    w_hh = [ts[3 * l + 1] for l in range(4)]
    bias = [ts[3 * l + 2] for l in range(4)]
    w_lin, b_lin = ts[12], ts[13]
    _check(w_lin.dim() == 2, "linear_weight must be rank-2")
    B, T, I = (int(v) for v in x.shape)
    H, O = hidden_size, int(w_lin.shape[0])
    _check(int(w_lin.shape[1]) == H, "linear_weight must be [O, H]")
    for l in range(4):
        _check(bias[l].dim() == 1 and bias[l].numel() == 4 * H, f"bias_l{l} must be [4H]")
    lib = _lib.load()
    nbytes = ctypes.c_size_t(0)
    _lib.check(lib.plstm_ref4_workspace_size(B, T, I, H, O, ctypes.byref(nbytes)))
    ws = torch.empty(int(nbytes.value), dtype=torch.uint8, device=dev)
    out = torch.empty(B, O, dtype=torch.float16, device=dev)
    a_ih, k1 = _lib.ptr_array([t.data_ptr() for t in w_ih])
    a_hh, k2 = _lib.ptr_array([t.data_ptr() for t in w_hh])
    a_b, k3 = _lib.ptr_array([t.data_ptr() for t in bias])
    watcher = device_status(dev)
    watcher.poll()  # a device failure of an earlier forward surfaces here
    with torch.cuda.device(dev):
        rc = getattr(lib, fn_name)(x.data_ptr(), B, T, I, H, O, a_ih, a_hh, a_b, w_lin.data_ptr(),
                                   b_lin.data_ptr(), out.data_ptr(), ws.data_ptr(), ws.numel(), _stream(dev))
    _lib.check(rc)
    watcher.watch(ws, torch.cuda.current_stream(dev))
    return out


def persistent_lstm4_forward(x, weight_ih_l0, weight_hh_l0, bias_l0, weight_ih_l1, weight_hh_l1, bias_l1,
                             weight_ih_l2, weight_hh_l2, bias_l2, weight_ih_l3, weight_hh_l3, bias_l3,
                             linear_weight, linear_bias):
    """Native [4H, K] weights (bindings.cpp:155)."""
    _check(weight_ih_l0.dim() == 2, "weight_ih_l0 must be rank-2")
    _check(weight_hh_l0.dim() == 2, "weight_hh_l0 must be rank-2")
    _check(linear_weight.dim() == 2, "linear_weight must be rank-2")
    args = [weight_ih_l0, weight_hh_l0, bias_l0, weight_ih_l1, weight_hh_l1, bias_l1, weight_ih_l2, weight_hh_l2,
            bias_l2, weight_ih_l3, weight_hh_l3, bias_l3, linear_weight, linear_bias]
    H = int(weight_hh_l0.shape[1])
    for l in range(4):
        _check(tuple(args[3 * l + 1].shape) == (4 * H, H), f"weight_hh_l{l} must be [4H, H]")
        _check(args[3 * l].dim() == 2 and args[3 * l].shape[0] == 4 * H, f"weight_ih_l{l} must be [4H, K]")
    _check(weight_ih_l0.shape[1] == x.shape[-1], "weight_ih_l0 must be [4H, I]")
    return _ref4_call("plstm_persistent_lstm4_forward", x, args, hidden_size=H)


def persistent_lstm4_forward_packed(x, weight_ih_l0_t, weight_hh_l0_t, bias_l0, weight_ih_l1_t, weight_hh_l1_t,
                                    bias_l1, weight_ih_l2_t, weight_hh_l2_t, bias_l2, weight_ih_l3_t,
                                    weight_hh_l3_t, bias_l3, linear_weight, linear_bias):
    """Transposed [K, 4H] weights (bindings.cpp:156)."""
    args = [weight_ih_l0_t, weight_hh_l0_t, bias_l0, weight_ih_l1_t, weight_hh_l1_t, bias_l1, weight_ih_l2_t,
            weight_hh_l2_t, bias_l2, weight_ih_l3_t, weight_hh_l3_t, bias_l3, linear_weight, linear_bias]
    _check(weight_hh_l0_t.dim() == 2, "weight_hh_l0_t must be rank-2")
    H = int(weight_hh_l0_t.shape[0])
    for l in range(4):
        _check(tuple(args[3 * l + 1].shape) == (H, 4 * H), f"weight_hh_l{l}_t must be [H, 4H]")
        _check(args[3 * l].dim() == 2 and args[3 * l].shape[1] == 4 * H, f"weight_ih_l{l}_t must be [K, 4H]")
    _check(weight_ih_l0_t.shape[0] == x.shape[-1], "weight_ih_l0_t must be [I, 4H]")
    return _ref4_call("plstm_persistent_lstm4_forward_packed", x, args, hidden_size=H)


def _kpair_args(x, args, ih_kpair: bool):
    _check(args[1].dim() == 3, "interleaved packed weight must be rank-3")
    rows = int(args[1].shape[1])
    H = rows // 4
    for l in range(4):
        _check(args[3 * l + 1].dim() == 3 and tuple(args[3 * l + 1].shape) == ((H + 1) // 2, 4 * H, 2),
               f"weight_hh_l{l} packed must be [ceil(H/2), 4H, 2]")
        if ih_kpair:
            k = int(x.shape[-1]) if l == 0 else H
            _check(args[3 * l].dim() == 3 and tuple(args[3 * l].shape) == ((k + 1) // 2, 4 * H, 2),
                   f"weight_ih_l{l} packed must be [ceil(K/2), 4H, 2]")
        else:
            k = int(x.shape[-1]) if l == 0 else H
            _check(tuple(args[3 * l].shape) == (4 * H, k), f"weight_ih_l{l} must be [4H, K]")
    return H


def persistent_lstm4_forward_interleaved(x, weight_ih_l0_packed, weight_hh_l0_packed, bias_l0,
                                         weight_ih_l1_packed, weight_hh_l1_packed, bias_l1, weight_ih_l2_packed,
                                         weight_hh_l2_packed, bias_l2, weight_ih_l3_packed, weight_hh_l3_packed,
                                         bias_l3, linear_weight, linear_bias):
    """k-pair packed W_ih and W_hh (bindings.cpp:157; the reference's default B=512 path)."""
    args = [weight_ih_l0_packed, weight_hh_l0_packed, bias_l0, weight_ih_l1_packed, weight_hh_l1_packed, bias_l1,
            weight_ih_l2_packed, weight_hh_l2_packed, bias_l2, weight_ih_l3_packed, weight_hh_l3_packed, bias_l3,
            linear_weight, linear_bias]
    H = _kpair_args(x, args, True)
    return _ref4_call("plstm_persistent_lstm4_forward_interleaved", x, args, hidden_size=H)


def persistent_lstm4_forward_monolithic(x, weight_ih_l0_packed, weight_hh_l0_packed, bias_l0,
                                        weight_ih_l1_packed, weight_hh_l1_packed, bias_l1, weight_ih_l2_packed,
                                        weight_hh_l2_packed, bias_l2, weight_ih_l3_packed, weight_hh_l3_packed,
                                        bias_l3, linear_weight, linear_bias):
    """k-pair packed weights, all layers in one kernel (bindings.cpp:162)."""
    args = [weight_ih_l0_packed, weight_hh_l0_packed, bias_l0, weight_ih_l1_packed, weight_hh_l1_packed, bias_l1,
            weight_ih_l2_packed, weight_hh_l2_packed, bias_l2, weight_ih_l3_packed, weight_hh_l3_packed, bias_l3,
            linear_weight, linear_bias]
    H = _kpair_args(x, args, True)
    return _ref4_call("plstm_persistent_lstm4_forward_monolithic", x, args, hidden_size=H)


def persistent_lstm4_forward_projected(x, weight_ih_l0, weight_hh_l0_packed, bias_l0, weight_ih_l1,
                                       weight_hh_l1_packed, bias_l1, weight_ih_l2, weight_hh_l2_packed, bias_l2,
                                       weight_ih_l3, weight_hh_l3_packed, bias_l3, linear_weight, linear_bias):
    """Native W_ih, k-pair packed W_hh (bindings.cpp:158)."""
    args = [weight_ih_l0, weight_hh_l0_packed, bias_l0, weight_ih_l1, weight_hh_l1_packed, bias_l1, weight_ih_l2,
            weight_hh_l2_packed, bias_l2, weight_ih_l3, weight_hh_l3_packed, bias_l3, linear_weight, linear_bias]
    H = _kpair_args(x, args, False)
    return _ref4_call("plstm_persistent_lstm4_forward_projected", x, args, hidden_size=H)


def _uniform(x, virtual_batch_size, args):
    # virtual_batch_size chose how many redundant DCU blocks computed the one
    # sequence (persistent_lstm_hip.cu:2399-2821); it does not change results.
    _check(int(virtual_batch_size) >= 1, "virtual_batch_size must be >= 1")
    return persistent_lstm4_forward_projected(x, *args)


def persistent_lstm4_forward_projected_uniform(x, virtual_batch_size, *args):
    """bindings.cpp:159."""
    return _uniform(x, virtual_batch_size, args)


def persistent_lstm4_forward_projected_uniform_p4(x, virtual_batch_size, *args):
    """bindings.cpp:160."""
    return _uniform(x, virtual_batch_size, args)


def persistent_lstm4_forward_projected_uniform_p8(x, virtual_batch_size, *args):
    """bindings.cpp:161."""
    return _uniform(x, virtual_batch_size, args)


def persistent_lstm_regressor_forward_generic_projected(x, weight_ih: Sequence[torch.Tensor],
                                                        weight_hh: Sequence[torch.Tensor],
                                                        bias: Sequence[torch.Tensor], linear_weight,
                                                        linear_bias):
    """Any number of layers, native weights, pre-summed bias (bindings.cpp:163)."""
    _check(isinstance(x, torch.Tensor) and x.dim() == 3, "x must be [B, T, I]")
    L = len(weight_ih)
    _check(L >= 1 and len(weight_hh) == L and len(bias) == L, "weight lists must have the same length >= 1")
    dev = x.device
    x = _cuda_f16(x, "x", dev)
    w_ih = [_cuda_f16(t, f"weight_ih[{i}]", dev) for i, t in enumerate(weight_ih)]
    w_hh = [_cuda_f16(t, f"weight_hh[{i}]", dev) for i, t in enumerate(weight_hh)]
    bs = [_cuda_f16(t, f"bias[{i}]", dev) for i, t in enumerate(bias)]
    w_lin = _cuda_f16(linear_weight, "linear_weight", dev)
    b_lin = _cuda_f16(linear_bias, "linear_bias", dev)
    B, T, I = (int(v) for v in x.shape)
    H = int(w_hh[0].shape[1])
    O = int(w_lin.shape[0])
    for l in range(L):
        _check(tuple(w_hh[l].shape) == (4 * H, H), f"weight_hh[{l}] must be [4H, H]")
        _check(tuple(w_ih[l].shape) == (4 * H, I if l == 0 else H), f"weight_ih[{l}] must be [4H, K]")
        _check(bs[l].numel() == 4 * H, f"bias[{l}] must be [4H]")
    from .core import PackedWeights
    pw = PackedWeights(w_ih, w_hh, bs, None, w_lin, b_lin, out_mode="last")
    out, _, _ = pw.forward(x, need_state=False)
    return out


def repeat_first_row(input: torch.Tensor, output_batch_size: int) -> torch.Tensor:
    """output[r] = input[0] for r < output_batch_size (bindings.cpp:164)."""
    _check(input.dim() == 2 and input.size(0) >= 1, "input must be [rows >= 1, cols]")
    if not input.is_cuda:
        raise ValueError("input must be a CUDA tensor")
    dt = {torch.float32: _lib.F32, torch.float16: _lib.F16, torch.bfloat16: _lib.BF16}.get(input.dtype)
    _check(dt is not None, "input must be float32, float16 or bfloat16")
    src = input.contiguous()
    rows = int(output_batch_size)
    out = torch.empty(rows, src.size(1), dtype=src.dtype, device=src.device)
    lib = _lib.load()
    with torch.cuda.device(src.device):
        _lib.check(lib.plstm_repeat_first_row(src.data_ptr(), int(src.size(1)), rows, dt, out.data_ptr(),
                                              _stream(src.device)))
    return out
