"""Shared pytest configuration: the `gpu` marker and fixture helpers."""
from __future__ import annotations

import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def load_golden(name: str) -> dict:
    with np.load(os.path.join(GOLDEN, name + ".npz")) as z:
        return {k: z[k] for k in z.files}


def golden_weights(g: dict, L: int):
    w_ih = [g[f"weight_ih_l{l}"] for l in range(L)]
    w_hh = [g[f"weight_hh_l{l}"] for l in range(L)]
    b_ih = [g[f"bias_ih_l{l}"] for l in range(L)]
    b_hh = [g[f"bias_hh_l{l}"] for l in range(L)]
    return w_ih, w_hh, b_ih, b_hh, g["linear_weight"], g["linear_bias"]


@pytest.fixture(scope="session")
def cuda_device():
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda:0")
