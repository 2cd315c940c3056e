"""Module-conversion API behaviour that needs no GPU: unsupported modules and
CPU inputs raise (no fallback), import aliases resolve."""
from __future__ import annotations

import sys

import pytest
import torch
import torch.nn as nn

import persistent_lstm_hip_b200 as plstm
from persistent_lstm_hip_b200 import ext


class M(nn.Module):
    def __init__(self, **kw):
        super().__init__()
        self.lstm = nn.LSTM(5, 16, 2, **kw)
        self.linear = nn.Linear(16, 3)


@pytest.mark.parametrize("kw", [dict(batch_first=False), dict(batch_first=True, bidirectional=True),
                                dict(batch_first=True, proj_size=8), dict(batch_first=True, bias=False)])
def test_unsupported_lstm_raises(kw):
    with pytest.raises(ValueError):
        plstm.convert_regressor_module(M(**kw))


def test_missing_submodules_raise():
    with pytest.raises(ValueError):
        plstm.convert_regressor_module(nn.Linear(3, 3))


def test_cpu_input_raises_instead_of_falling_back():
    conv = plstm.convert_regressor_module(M(batch_first=True))
    assert isinstance(conv, plstm.PersistentLSTMRegressor)
    with pytest.raises(ValueError, match="CUDA"):
        conv(torch.randn(2, 4, 5))
    lstm = plstm.convert_lstm_module(nn.LSTM(5, 16, 1, batch_first=True))
    with pytest.raises(ValueError, match="CUDA"):
        lstm(torch.randn(2, 4, 5))


def test_ext_rejects_cpu_and_bad_shapes():
    w = [torch.zeros(512, 5, dtype=torch.float16)] + [torch.zeros(1)] * 13
    with pytest.raises(ValueError):
        ext.persistent_lstm4_forward(torch.zeros(2, 3, dtype=torch.float16), *w)
    with pytest.raises(ValueError):
        ext.repeat_first_row(torch.zeros(1, 3), 4)


def test_backend_env_validation(monkeypatch):
    conv = plstm.convert_regressor_module(M(batch_first=True))
    monkeypatch.setenv("PERSISTENT_LSTM_HIP_BACKEND", "bogus")
    with pytest.raises(ValueError):
        conv._forced_backend()


def test_replace_lstm_inplace_and_copy():
    m = nn.Sequential(nn.LSTM(5, 16, 1, batch_first=True))
    c = plstm.convert_model_copy(m)
    assert isinstance(c[0], plstm.PersistentLSTM) and isinstance(m[0], nn.LSTM)
    plstm.replace_lstm_inplace(m)
    assert isinstance(m[0], plstm.PersistentLSTM)
    torch.testing.assert_close(m[0].weight_hh_l0, c[0].weight_hh_l0)


def test_install_aliases():
    plstm.install_aliases()
    import persistent_lstm_hip  # noqa: F401
    import persistent_lstm_hip_ext  # noqa: F401
    assert sys.modules["persistent_lstm_hip"].convert_regressor_module is plstm.convert_regressor_module
    assert hasattr(sys.modules["persistent_lstm_hip_ext"], "persistent_lstm4_forward_interleaved")
