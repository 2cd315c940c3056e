"""Shared helpers of the parity tests: seeded models, inputs and the oracle call."""
from __future__ import annotations

import numpy as np
import torch
import torch.nn as nn

from oracle import oracle

# North-star tolerances for the 16-bit paths and the f32 path.
TOL16_MAX, TOL16_MEAN = 2e-2, 5e-3
TOL32_MAX = 1e-4


class Regressor(nn.Module):
    def __init__(self, I, H, L, O):
        super().__init__()
        self.lstm = nn.LSTM(I, H, L, batch_first=True)
        self.linear = nn.Linear(H, O)


def make_model(I, H, L, O, seed=0):
    torch.manual_seed(seed)
    return Regressor(I, H, L, O).eval()


def weights_of(m, L, dtype, device):
    f = lambda t: t.detach().to(device=device, dtype=dtype).contiguous()
    w_ih = [f(getattr(m.lstm, f"weight_ih_l{l}")) for l in range(L)]
    w_hh = [f(getattr(m.lstm, f"weight_hh_l{l}")) for l in range(L)]
    b_ih = [f(getattr(m.lstm, f"bias_ih_l{l}")) for l in range(L)]
    b_hh = [f(getattr(m.lstm, f"bias_hh_l{l}")) for l in range(L)]
    return w_ih, w_hh, b_ih, b_hh, f(m.linear.weight), f(m.linear.bias)


def np64(t):
    return None if t is None else t.detach().to("cpu", torch.float64).numpy()


def oracle_of(x, w_ih, w_hh, b_ih, b_hh, w_lin, b_lin, *, lengths=None, hx=None, out_mode="seq", rows=None):
    """Runs the f64 oracle on exactly the (rounded) values the device saw;
    `rows` restricts it to a subset of batch rows."""
    xs = np64(x)
    lens = None if lengths is None else lengths.detach().cpu().numpy().astype(np.int32)
    h0 = c0 = None
    if hx is not None:
        h0, c0 = np64(hx[0]), np64(hx[1])
    if rows is not None:
        xs = xs[rows]
        lens = None if lens is None else lens[rows]
        if h0 is not None:
            h0, c0 = h0[:, rows], c0[:, rows]
    return oracle.forward(xs, [np64(w) for w in w_ih], [np64(w) for w in w_hh], [np64(b) for b in b_ih],
                          [np64(b) for b in b_hh], np64(w_lin), np64(b_lin), lengths=lens, h0=h0, c0=c0,
                          out_mode=out_mode)


def assert_close16(got, ref, what=""):
    g = got.detach().to("cpu", torch.float64).numpy() if isinstance(got, torch.Tensor) else got
    diff = np.abs(g - ref)
    mx, mean = float(diff.max()) if diff.size else 0.0, float(diff.mean()) if diff.size else 0.0
    assert mx <= TOL16_MAX and mean <= TOL16_MEAN, f"{what}: max_abs={mx:.3g} mean_abs={mean:.3g}"
    return mx, mean


def assert_close32(got, ref, what=""):
    g = got.detach().to("cpu", torch.float64).numpy()
    diff = np.abs(g - ref)
    mx = float(diff.max()) if diff.size else 0.0
    assert mx <= TOL32_MAX, f"{what}: max_abs={mx:.3g}"
    return mx
