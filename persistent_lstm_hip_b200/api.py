"""Module conversion functions (persistent_lstm_hip/persistent_lstm_hip/api.py:10-43)."""
from __future__ import annotations

import copy

import torch.nn as nn

from .model import PersistentLSTM, PersistentLSTMRegressor
from .packing import check_lstm_supported


def convert_lstm_module(lstm: nn.LSTM) -> PersistentLSTM:
    return PersistentLSTM.from_native_module(lstm)


def convert_regressor_module(model: nn.Module) -> PersistentLSTMRegressor:
    """model.lstm (nn.LSTM) + model.linear (nn.Linear) -> PersistentLSTMRegressor.

    Raises ValueError where the reference would have returned its
    native-PyTorch fallback wrapper (api.py:14-29): this package has no
    fallback, and every batch-first, unidirectional, projection-free LSTM with
    biases runs on the CUDA library (tensor-core kernel for H = 128, L <= 4,
    f16/bf16; the generic kernel otherwise).
    """
    if not hasattr(model, "lstm") or not hasattr(model, "linear"):
        raise ValueError("convert_regressor_module needs a model with `.lstm` and `.linear`")
    if not isinstance(model.lstm, nn.LSTM):
        raise ValueError("model.lstm must be an nn.LSTM")
    if not isinstance(model.linear, nn.Linear):
        raise ValueError("model.linear must be an nn.Linear")
    check_lstm_supported(model.lstm)
    if model.linear.in_features != model.lstm.hidden_size:
        raise ValueError("model.linear.in_features must equal model.lstm.hidden_size")
    return PersistentLSTMRegressor.from_native_module(model)


def replace_lstm_inplace(model: nn.Module) -> nn.Module:
    for name, child in list(model.named_children()):
        if isinstance(child, nn.LSTM):
            setattr(model, name, PersistentLSTM.from_native_module(child))
        else:
            replace_lstm_inplace(child)
    return model


def convert_model_copy(model: nn.Module) -> nn.Module:
    return replace_lstm_inplace(copy.deepcopy(model))
