"""Drop-in for the reference's `miopen_adaptive_lstm_hip` package API
(miopen_adaptive_lstm_hip/miopen_adaptive_lstm_hip/__init__.py:14, api.py:1-7):
`AdaptiveLSTMRegressor(native_module)`, `convert_regressor_module`,
`NativeModuleFallback`, and `_C` (the extension's functions, ``adaptive_ext``).

The reference's regressor picks among its MIOpen-style HIP backends per layer
(model.py:596-1091: input GEMM, then one of its hidden-update kernels, then the
Linear head) and returns its native PyTorch module's output for CPU tensors,
training mode or non-FP16 inputs.  Here the whole forward is the single CUDA
path (the fused tensor-core kernels, or the FFMA kernel for shapes they do not
serve); it raises instead of falling back.  Its planner objects (scheduler,
descriptors, modular pipeline) only chose among the HIP kernels and are not
provided.
"""
from __future__ import annotations

import copy

import torch
import torch.nn as nn

from . import adaptive_ext as _C  # noqa: N812  (the reference's extension name)
from .model import NativeModuleFallback, PersistentLSTMRegressor
from .packing import check_lstm_supported, pack_regressor_module

__all__ = ["AdaptiveLSTMRegressor", "NativeModuleFallback", "convert_regressor_module", "_C"]


class AdaptiveLSTMRegressor(PersistentLSTMRegressor):
    """`nn.LSTM + nn.Linear` regressor (reference model.py:347-1091): forward(x) -> [B, O],
    the Linear head on the last step, computed by this library's CUDA path."""

    def __init__(self, native_module: nn.Module):
        if not hasattr(native_module, "lstm") or not hasattr(native_module, "linear"):
            raise ValueError("AdaptiveLSTMRegressor needs a module with `.lstm` and `.linear`")
        check_lstm_supported(native_module.lstm)
        super().__init__(pack_regressor_module(copy.deepcopy(native_module)))
        self.train(native_module.training)  # the wrapped module's mode, as the reference's copy keeps it

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.training:
            raise RuntimeError("AdaptiveLSTMRegressor is inference-only: call .eval() (the reference fell back "
                               "to its PyTorch module here)")
        return super().forward(x)


def convert_regressor_module(model: nn.Module) -> AdaptiveLSTMRegressor:
    """model.lstm + model.linear -> AdaptiveLSTMRegressor (reference model.py convert_regressor_module);
    raises ValueError where the reference returned NativeModuleFallback."""
    if not isinstance(getattr(model, "lstm", None), nn.LSTM) or not isinstance(getattr(model, "linear", None),
                                                                              nn.Linear):
        raise ValueError("convert_regressor_module needs `.lstm` (nn.LSTM) and `.linear` (nn.Linear)")
    if model.linear.in_features != model.lstm.hidden_size:
        raise ValueError("model.linear.in_features must equal model.lstm.hidden_size")
    return AdaptiveLSTMRegressor(model)
