"""nn.Module wrappers with the reference's class names and call signatures.

Mirrors persistent_lstm_hip/persistent_lstm_hip/model.py:
  * StandardLSTMRegressor          :30-45   (plain PyTorch model definition)
  * NativeModuleFallback           :48-320  (explicit opt-in wrapper only)
  * PersistentLSTM                 :323-395 (nn.LSTM-compatible forward)
  * PersistentLSTMRegressor        :398-658 (the fused LSTM + Linear forward)
Every forward of PersistentLSTM / PersistentLSTMRegressor runs the CUDA
library; a CPU input raises instead of falling back.
"""
from __future__ import annotations

import os
from typing import Any, Optional, Tuple

import torch
import torch.nn as nn

from . import core
from .packing import PackedLSTMLayerWeights, PackedLSTMWeights, PackedRegressorWeights, pack_lstm_module, \
    pack_regressor_module

_OFF = {"0", "false", "no", "off", "disable", "disabled"}
_ON = {"1", "true", "yes", "on", "force", "forced", "assume"}
_AUTO = {"", "auto", "detect"}
_DEDUPE = {"dedupe", "rows"}


class StandardLSTMRegressor(nn.Module):
    """nn.LSTM(batch_first) + Linear on the last step (the reference's LSTMRegressor)."""

    def __init__(self, input_dim: int, hidden_dim: int, output_dim: int, n_layers: int, dropout: float = 0.2):
        super().__init__()
        self.lstm = nn.LSTM(input_dim, hidden_dim, n_layers, batch_first=True, dropout=dropout)
        self.linear = nn.Linear(hidden_dim, output_dim)
        self.dropout = nn.Dropout(dropout)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        out, _ = self.lstm(x)
        return self.linear(self.dropout(out[:, -1, :]))


class NativeModuleFallback(nn.Module):
    """Runs a wrapped PyTorch module unchanged.

    Kept for API compatibility with the reference (model.py:48-320).  None of
    this package's conversion functions returns it: shapes the CUDA library
    cannot serve raise instead.
    """

    def __init__(self, native_module: nn.Module, backend_name: str = "native_pytorch_generic",
                 enable_uniform_batch: bool = False):
        super().__init__()
        self.module = native_module
        self._backend_name = backend_name
        self._enable_uniform_batch = enable_uniform_batch

    @property
    def backend_name(self) -> str:
        return self._backend_name

    def forward(self, *args: Any, **kwargs: Any) -> Any:
        return self.module(*args, **kwargs)


def _param_key(tensors) -> tuple:
    key = []
    for t in tensors:
        key.extend((id(t), t.device.type, t.device.index, str(t.dtype), tuple(t.shape), t._version))
    return tuple(key)


class PersistentLSTM(nn.Module):
    """nn.LSTM(batch_first=True)-compatible module on the CUDA kernels.

    forward(x, hx=None, lengths=None) -> (out[B,T,H], (h_n, c_n)); with
    `lengths` the semantics are those of pack_padded_sequence (state frozen
    after each length, outputs zero past it).
    """

    def __init__(self, packed: PackedLSTMWeights):
        super().__init__()
        self.input_size = packed.input_size
        self.hidden_size = packed.hidden_size
        self.num_layers = packed.num_layers
        self.batch_first = packed.batch_first
        self.bidirectional = False
        self.proj_size = 0
        for l, layer in enumerate(packed.layers):
            setattr(self, f"weight_ih_l{l}", nn.Parameter(layer.weight_ih.detach().clone()))
            setattr(self, f"weight_hh_l{l}", nn.Parameter(layer.weight_hh.detach().clone()))
            setattr(self, f"bias_ih_l{l}", nn.Parameter(layer.bias_ih.detach().clone()))
            setattr(self, f"bias_hh_l{l}", nn.Parameter(layer.bias_hh.detach().clone()))
        self._cache_key = None
        self._cache: Optional[core.PackedWeights] = None

    @classmethod
    def from_native_module(cls, lstm: nn.LSTM) -> "PersistentLSTM":
        return cls(pack_lstm_module(lstm))

    def _params(self):
        out = []
        for l in range(self.num_layers):
            out += [getattr(self, f"weight_ih_l{l}"), getattr(self, f"weight_hh_l{l}"),
                    getattr(self, f"bias_ih_l{l}"), getattr(self, f"bias_hh_l{l}")]
        return out

    def _packed(self) -> PackedLSTMWeights:
        return PackedLSTMWeights(
            self.input_size, self.hidden_size, self.num_layers, self.batch_first,
            [PackedLSTMLayerWeights(getattr(self, f"weight_ih_l{l}"), getattr(self, f"weight_hh_l{l}"),
                                    getattr(self, f"bias_ih_l{l}"), getattr(self, f"bias_hh_l{l}"))
             for l in range(self.num_layers)])

    @property
    def backend_name(self) -> str:
        p = self._params()[0]
        return "b200_" + core.select_backend(input_size=self.input_size, hidden_size=self.hidden_size,
                                             num_layers=self.num_layers, output_size=1, dtype=p.dtype,
                                             out_mode="hseq", device=p.device.index or 0)

    def can_use_specialized_hip(self) -> bool:
        return True

    def packed_weights(self) -> core.PackedWeights:
        params = self._params()
        key = _param_key(params)
        if self._cache is None or self._cache_key != key:
            L = self.num_layers
            with torch.no_grad():
                self._cache = core.PackedWeights(
                    [params[4 * l] for l in range(L)], [params[4 * l + 1] for l in range(L)],
                    [params[4 * l + 2] for l in range(L)], [params[4 * l + 3] for l in range(L)],
                    None, None, out_mode="hseq")
            self._cache_key = key
        return self._cache

    def forward(self, x: torch.Tensor, hx: Optional[Tuple[torch.Tensor, torch.Tensor]] = None,
                lengths: Optional[torch.Tensor] = None):
        with torch.no_grad():
            out, h_n, c_n = self.packed_weights().forward(x, lengths=lengths, hx=hx)
        return out, (h_n, c_n)


class PersistentLSTMRegressor(nn.Module):
    """The fused LSTM + Linear regressor forward (reference model.py:398-658).

    forward(x) -> [B, O]: Linear on each row's last step, like the reference.
    forward_sequence(x, lengths=None, hx=None) -> (out[B,T,O], (h_n, c_n)).
    """

    def __init__(self, packed: PackedRegressorWeights):
        super().__init__()
        self.lstm = PersistentLSTM(packed.lstm)
        self.linear = nn.Linear(packed.linear_weight.shape[1], packed.linear_weight.shape[0])
        with torch.no_grad():
            self.linear.weight.copy_(packed.linear_weight)
            self.linear.bias.copy_(packed.linear_bias)
        self.linear.to(device=packed.linear_weight.device, dtype=packed.linear_weight.dtype)
        self._cache = {}
        self._uniform_key = None
        self._uniform_value = False
        self._debug_reported = False

    @classmethod
    def from_native_module(cls, native_module: nn.Module) -> "PersistentLSTMRegressor":
        return cls(pack_regressor_module(native_module))

    def _packed(self) -> PackedRegressorWeights:
        return PackedRegressorWeights(self.lstm._packed(), self.linear.weight, self.linear.bias)

    def _can_use_specialized_regressor_hip(self) -> bool:
        return True

    @property
    def backend_name(self) -> str:
        forced = self._forced_backend()
        p = self.linear.weight
        b = core.select_backend(input_size=self.lstm.input_size, hidden_size=self.lstm.hidden_size,
                                num_layers=self.lstm.num_layers, output_size=self.linear.out_features,
                                dtype=p.dtype, out_mode="last", device=p.device.index or 0)
        return f"b200_{b}_regressor[{forced}]"

    @staticmethod
    def _forced_backend() -> str:
        # PERSISTENT_LSTM_HIP_BACKEND chose among the reference's DCU kernels
        # (model.py:477-491); every value maps to the single CUDA path here.
        forced = os.environ.get("PERSISTENT_LSTM_HIP_BACKEND", "auto").strip().lower()
        if forced not in {"", "auto", "interleaved", "projected", "monolithic"}:
            raise ValueError("PERSISTENT_LSTM_HIP_BACKEND must be one of: auto, interleaved, projected, monolithic")
        return forced or "auto"

    def packed_weights(self, out_mode: str) -> core.PackedWeights:
        params = self.lstm._params() + [self.linear.weight, self.linear.bias]
        key = (out_mode, _param_key(params))
        hit = self._cache.get(out_mode)
        if hit is None or hit[0] != key:
            L = self.lstm.num_layers
            with torch.no_grad():
                pw = core.PackedWeights(
                    [params[4 * l] for l in range(L)], [params[4 * l + 1] for l in range(L)],
                    [params[4 * l + 2] for l in range(L)], [params[4 * l + 3] for l in range(L)],
                    self.linear.weight, self.linear.bias, out_mode=out_mode)
            self._cache[out_mode] = (key, pw)
            hit = self._cache[out_mode]
        return hit[1]

    def _uniform_batch(self, x: torch.Tensor) -> bool:
        """Optional duplicate-row shortcut of the reference (model.py:493-520):
        with PERSISTENT_LSTM_HIP_UNIFORM_BATCH=auto, a batch whose rows are all
        identical is computed once and broadcast.  Off by default here because
        the detection costs a full pass over x and a host synchronisation.
        The value "dedupe" selects the general form instead (any set of
        identical rows computed once, on the GPU; `_dedupe_rows`)."""
        mode = os.environ.get("PERSISTENT_LSTM_HIP_UNIFORM_BATCH", "0").strip().lower()
        if mode in _OFF or mode in _DEDUPE or x.dim() != 3 or x.size(0) <= 1:
            return False
        if mode in _ON:
            return True
        if mode not in _AUTO:
            raise ValueError("PERSISTENT_LSTM_HIP_UNIFORM_BATCH must be one of: auto, detect, assume, dedupe, 1, 0")
        key = (x.data_ptr(), x.device.index, str(x.dtype), tuple(x.shape), tuple(x.stride()), x._version)
        if self._uniform_key != key:
            self._uniform_value = bool(torch.equal(x, x.narrow(0, 0, 1).expand_as(x)))
            self._uniform_key = key
        return self._uniform_value

    @staticmethod
    def _dedupe_rows() -> bool:
        mode = os.environ.get("PERSISTENT_LSTM_HIP_UNIFORM_BATCH", "0").strip().lower()
        return mode in _DEDUPE

    def forward(self, x: torch.Tensor, lengths: Optional[torch.Tensor] = None) -> torch.Tensor:
        self._forced_backend()
        dedupe = self._dedupe_rows()
        uniform = lengths is None and self._uniform_batch(x)
        xin = x.narrow(0, 0, 1) if uniform else x
        pw = self.packed_weights("last")
        if os.environ.get("PERSISTENT_LSTM_HIP_DEBUG", "0") == "1" and not self._debug_reported:
            print(f"persistent_lstm_hip_b200 debug: backend={pw.backend}, batch={int(x.size(0))}, "
                  f"seq_len={int(x.size(1))}, uniform_batch_fast_path={uniform}, dedupe_rows={dedupe}")
            self._debug_reported = True
        with torch.no_grad():
            out, _, _ = pw.forward(xin, lengths=lengths, need_state=False, dedupe=dedupe)
        if uniform:
            from .ext import repeat_first_row
            return repeat_first_row(out, int(x.size(0)))
        return out

    def forward_sequence(self, x: torch.Tensor, lengths: Optional[torch.Tensor] = None,
                         hx: Optional[Tuple[torch.Tensor, torch.Tensor]] = None):
        with torch.no_grad():
            out, h_n, c_n = self.packed_weights("seq").forward(x, lengths=lengths, hx=hx,
                                                               dedupe=self._dedupe_rows())
        return out, (h_n, c_n)


PersistentLSTM4LayerRegressor = PersistentLSTMRegressor
