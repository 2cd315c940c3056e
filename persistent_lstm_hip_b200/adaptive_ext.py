"""Drop-in for functions of the reference's `miopen_adaptive_lstm_hip._C` extension.

Mirrors miopen_adaptive_lstm_hip/csrc/bindings.cpp:5-78 function by function
as thin torch-tensor shims over the C ABI (include/plstm.h).
"""
from __future__ import annotations

import torch

from . import _lib
from .core import _stream

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
