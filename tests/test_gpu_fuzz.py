"""Seeded randomized parity sweep: shapes drawn across every backend's envelope.

Each case draws batch, length, input, hidden and layer sizes, dtype, output mode,
variable lengths and an initial state, runs the library's forward, and checks
out / h_n / c_n against the f64 oracle at the north-star tolerances (16-bit:
max 2e-2, mean 5e-3; f32: max 1e-4).
- 16-bit cases run on the default backend choice: the tensor-core wavefront kernel
  for H <= 128, the tensor-core layer path up to H = 512, and the FFMA kernel beyond
  the envelope (I > 128).
- Every fourth 16-bit case also forces the FFMA kernel.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from helpers import assert_close16, assert_close32, make_model, oracle_of, weights_of
import persistent_lstm_hip_b200 as plstm

pytestmark = pytest.mark.gpu

_H = [1, 7, 33, 64, 100, 128, 130, 192, 256, 300]
_I = [1, 3, 5, 16, 40, 127, 128, 140]


def _case(seed):
    r = np.random.default_rng(1000 + seed)
    return dict(
        B=int(r.integers(1, 71)), T=int(r.integers(1, 25)), I=int(r.choice(_I)), H=int(r.choice(_H)),
        L=int(r.integers(1, 6)), O=int(r.integers(1, 33)),
        dtype=[torch.float16, torch.bfloat16, torch.float32][int(r.integers(0, 3))],
        mode=["seq", "last", "hseq"][int(r.integers(0, 3))],
        varlen=bool(r.integers(0, 2)), state=bool(r.integers(0, 2)))


@pytest.mark.parametrize("seed", range(32))
def test_random_shape_matches_oracle(cuda_device, seed):
    c = _case(seed)
    B, T, I, H, L, O, dt = c["B"], c["T"], c["I"], c["H"], c["L"], c["O"], c["dtype"]
    m = make_model(I, H, L, O, seed=seed)
    w = weights_of(m, L, dt, cuda_device)
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(B, T, I, generator=g).to(cuda_device, dt)
    lens = None
    if c["varlen"]:
        lens = torch.randint(1, T + 1, (B,), generator=g, dtype=torch.int32)
        lens[0] = T
    hx = None
    if c["state"]:
        hx = tuple((0.5 * torch.randn(L, B, H, generator=g)).to(cuda_device, dt) for _ in range(2))
    backends = ["auto"]
    if dt != torch.float32 and seed % 4 == 0:
        backends.append("simt")
    ref = oracle_of(x, *w, lengths=lens, hx=hx, out_mode=c["mode"])
    for be in backends:
        out, h_n, c_n = plstm.lstm_linear_forward(x, *w, lengths=lens, hx=hx, out_mode=c["mode"], backend=be,
                                                  check=True)
        close = assert_close32 if dt == torch.float32 else assert_close16
        what = f"{be} {c}"
        close(out, ref[0], f"out {what}")
        close(h_n, ref[1], f"h_n {what}")
        close(c_n, ref[2], f"c_n {what}")
