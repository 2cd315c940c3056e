"""B200-native persistent LSTM + Linear inference path.

Drop-in for the fused `nn.LSTM + nn.Linear` forward of
mantuoluozk/persistent_lstm_hip: the module-conversion API of its
`persistent_lstm_hip` package (persistent_lstm_hip/persistent_lstm_hip/__init__.py:1-20)
and the functions of its `persistent_lstm_hip_ext` extension (``ext``), on a
torch-free CUDA library with a C ABI (include/plstm.h, lib/libplstm.so).

``install_aliases()`` registers this package under the reference's import
names so unmodified reference-style code (``from persistent_lstm_hip import
convert_regressor_module``, ``from miopen_adaptive_lstm_hip import
AdaptiveLSTMRegressor``, ``miopen_adaptive_lstm_hip._C``) runs on it.
"""
from __future__ import annotations

import sys

from . import adaptive, adaptive_ext, ext
from ._lib import PlstmError, PlstmUnavailable
from .api import convert_lstm_module, convert_model_copy, convert_regressor_module, replace_lstm_inplace
from .core import PackedWeights, check_device_status, lstm_linear_forward, select_backend, unique_rows
from .model import (NativeModuleFallback, PersistentLSTM, PersistentLSTM4LayerRegressor, PersistentLSTMRegressor,
                    StandardLSTMRegressor)

__all__ = [
    "PersistentLSTM",
    "PersistentLSTMRegressor",
    "PersistentLSTM4LayerRegressor",
    "NativeModuleFallback",
    "StandardLSTMRegressor",
    "convert_lstm_module",
    "convert_regressor_module",
    "replace_lstm_inplace",
    "convert_model_copy",
    "lstm_linear_forward",
    "PackedWeights",
    "select_backend",
    "unique_rows",
    "check_device_status",
    "PlstmError",
    "PlstmUnavailable",
    "ext",
    "adaptive",
    "adaptive_ext",
    "install_aliases",
]


def install_aliases() -> None:
    """Makes `import persistent_lstm_hip` and `import persistent_lstm_hip_ext`
    resolve to this package and its extension shim."""
    from . import api, model, packing

    pkg = sys.modules[__name__]
    sys.modules.setdefault("persistent_lstm_hip", pkg)
    sys.modules.setdefault("persistent_lstm_hip.api", api)
    sys.modules.setdefault("persistent_lstm_hip.model", model)
    sys.modules.setdefault("persistent_lstm_hip.packing", packing)
    sys.modules.setdefault("persistent_lstm_hip_ext", ext)
    sys.modules.setdefault("miopen_adaptive_lstm_hip", adaptive)
    sys.modules.setdefault("miopen_adaptive_lstm_hip.api", adaptive)
    sys.modules.setdefault("miopen_adaptive_lstm_hip._C", adaptive_ext)
