"""Weight containers and host-side layout helpers.

Mirrors persistent_lstm_hip/persistent_lstm_hip/packing.py (dataclasses and
module packing, :10-73) and the k-pair layout helpers the reference's wrappers
use: ``pack_recurrent_weight_kpairs`` restates ``_pack_recurrent_weight_kpairs``
(persistent_lstm_hip/model.py:20-27) and ``unpack_recurrent_weight_kpairs``
restates the inverse the C++ op applies before its CPU path
(persistent_lstm_hip/csrc/persistent_lstm_op.cpp:159-166).  The device kernels
never need these: plstm_pack reads native, transposed and k-pair layouts
directly.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import List

import torch
import torch.nn as nn


@dataclass
class PackedLSTMLayerWeights:
    weight_ih: torch.Tensor
    weight_hh: torch.Tensor
    bias_ih: torch.Tensor
    bias_hh: torch.Tensor

    @property
    def bias(self) -> torch.Tensor:
        return (self.bias_ih + self.bias_hh).contiguous()


@dataclass
class PackedLSTMWeights:
    input_size: int
    hidden_size: int
    num_layers: int
    batch_first: bool
    layers: List[PackedLSTMLayerWeights]


@dataclass
class PackedRegressorWeights:
    lstm: PackedLSTMWeights
    linear_weight: torch.Tensor
    linear_bias: torch.Tensor


def check_lstm_supported(lstm: nn.LSTM) -> None:
    """Raises ValueError for the nn.LSTM variants this path does not serve
    (the same ones the reference rejects, packing.py:39-44)."""
    if not lstm.batch_first:
        raise ValueError("only batch_first=True LSTMs are supported")
    if lstm.bidirectional:
        raise ValueError("only unidirectional LSTMs are supported")
    if lstm.proj_size != 0:
        raise ValueError("proj_size is not supported")
    if not lstm.bias:
        raise ValueError("bias=False LSTMs are not supported")


def pack_lstm_module(lstm: nn.LSTM) -> PackedLSTMWeights:
    check_lstm_supported(lstm)
    layers = [
        PackedLSTMLayerWeights(
            weight_ih=getattr(lstm, f"weight_ih_l{l}").contiguous(),
            weight_hh=getattr(lstm, f"weight_hh_l{l}").contiguous(),
            bias_ih=getattr(lstm, f"bias_ih_l{l}").contiguous(),
            bias_hh=getattr(lstm, f"bias_hh_l{l}").contiguous(),
        )
        for l in range(lstm.num_layers)
    ]
    return PackedLSTMWeights(lstm.input_size, lstm.hidden_size, lstm.num_layers, lstm.batch_first, layers)


def pack_regressor_module(native_module: nn.Module) -> PackedRegressorWeights:
    return PackedRegressorWeights(
        lstm=pack_lstm_module(native_module.lstm),
        linear_weight=native_module.linear.weight.contiguous(),
        linear_bias=native_module.linear.bias.contiguous(),
    )


def pack_recurrent_weight_kpairs(weight: torch.Tensor) -> torch.Tensor:
    """[4H, K] -> [ceil(K/2), 4H, 2]: element (r, k) lands at [k // 2, r, k % 2];
    an odd K gets one zero column."""
    wt = weight.transpose(0, 1)
    k, rows = wt.shape
    if k % 2:
        wt = torch.cat((wt, wt.new_zeros(1, rows)), dim=0)
        k += 1
    return wt.reshape(k // 2, 2, rows).permute(0, 2, 1).contiguous()


def unpack_recurrent_weight_kpairs(packed: torch.Tensor, original_k: int) -> torch.Tensor:
    """Inverse of pack_recurrent_weight_kpairs: [P, 4H, 2] -> [4H, original_k]."""
    if packed.dim() != 3 or packed.shape[2] != 2:
        raise ValueError("k-pair packed weight must be [P, 4H, 2]")
    pairs, rows, _ = packed.shape
    full = packed.permute(0, 2, 1).reshape(pairs * 2, rows)
    return full[:original_k].transpose(0, 1).contiguous()
