"""Test infrastructure only: Python front end of the CPU parity oracle.

Two restatements of the reference's LSTM + Linear forward
(persistent_lstm_hip/persistent_lstm_hip/reference.py:11-72,
persistent_lstm_hip/csrc/persistent_lstm_reference.cpp:7-64):

* ``forward``: the C oracle (plstm_oracle.c) through ctypes, f64 or f32,
  OpenMP over batch rows.  This is the checker of every parity test and the
  CPU baseline of bench.py.
* ``forward_numpy``: a vectorised numpy restatement used to cross-check the C
  oracle on small shapes.

Both take float numpy arrays in nn.LSTM's native layouts (W_ih[4H][I or H],
W_hh[4H][H], biases [4H], W_lin[O][H], b_lin[O]) and return
``(out, h_n, c_n)``.  ``out_mode`` is "seq" ([B,T,O], zero past each length),
"last" ([B,O] at each row's last valid step) or "hseq" (the last layer's h
sequence [B,T,H], no Linear).
"""
from __future__ import annotations

import ctypes
import os
from typing import Optional, Sequence

import numpy as np

from . import build as _build

_MODES = {"seq": 1, "last": 2, "hseq": 3}


class _Desc(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in (
        "batch", "seq_len", "input_size", "hidden_size", "num_layers", "output_size",
        "out_mode", "threads")]


_lib = None


def _load():
    global _lib
    if _lib is None:
        path = _build.LIB
        if not os.path.exists(path):
            path = _build.build()
        lib = ctypes.CDLL(path)
        for name, real in (("oracle_forward_f64", ctypes.c_double), ("oracle_forward_f32", ctypes.c_float)):
            fn = getattr(lib, name)
            p = ctypes.POINTER(real)
            pp = ctypes.POINTER(p)
            fn.argtypes = [ctypes.POINTER(_Desc), p, pp, pp, pp, pp, p, p,
                           ctypes.POINTER(ctypes.c_int32), p, p, p, p, p]
            fn.restype = ctypes.c_int
        lib.oracle_max_threads.restype = ctypes.c_int
        _lib = lib
    return _lib


def max_threads() -> int:
    return int(_load().oracle_max_threads())


def _ptr(a, real):
    if a is None:
        return None
    return a.ctypes.data_as(ctypes.POINTER(real))


def forward(x: np.ndarray, w_ih: Sequence[np.ndarray], w_hh: Sequence[np.ndarray],
            b_ih: Optional[Sequence[np.ndarray]], b_hh: Optional[Sequence[np.ndarray]],
            w_lin: Optional[np.ndarray], b_lin: Optional[np.ndarray], *,
            lengths: Optional[np.ndarray] = None, h0: Optional[np.ndarray] = None,
            c0: Optional[np.ndarray] = None, out_mode: str = "seq",
            precision: str = "f64", threads: int = 0):
    """Runs the C oracle.  Returns (out, h_n, c_n) as arrays of `precision`."""
    lib = _load()
    dt = np.float64 if precision == "f64" else np.float32
    real = ctypes.c_double if precision == "f64" else ctypes.c_float
    fn = lib.oracle_forward_f64 if precision == "f64" else lib.oracle_forward_f32
    x = np.ascontiguousarray(x, dtype=dt)
    B, T, I = x.shape
    L = len(w_ih)
    H = w_hh[0].shape[1]
    O = 0 if out_mode == "hseq" else int(w_lin.shape[0])
    keep = []

    def arr(a):
        a = np.ascontiguousarray(a, dtype=dt)
        keep.append(a)
        return a

    def plist(lst):
        if lst is None:
            return None
        ptrs = (ctypes.POINTER(real) * L)(*[_ptr(arr(a), real) if a is not None else None for a in lst])
        keep.append(ptrs)
        return ctypes.cast(ptrs, ctypes.POINTER(ctypes.POINTER(real)))

    d = _Desc(B, T, I, H, L, O, _MODES[out_mode], int(threads))
    if out_mode == "seq":
        out = np.zeros((B, T, O), dtype=dt)
    elif out_mode == "last":
        out = np.zeros((B, O), dtype=dt)
    else:
        out = np.zeros((B, T, H), dtype=dt)
    h_n = np.zeros((L, B, H), dtype=dt)
    c_n = np.zeros((L, B, H), dtype=dt)
    lens = None
    if lengths is not None:
        lens = np.ascontiguousarray(lengths, dtype=np.int32)
        keep.append(lens)
    rc = fn(ctypes.byref(d), _ptr(x, real), plist(w_ih), plist(w_hh), plist(b_ih), plist(b_hh),
            _ptr(arr(w_lin), real) if w_lin is not None and out_mode != "hseq" else None,
            _ptr(arr(b_lin), real) if b_lin is not None and out_mode != "hseq" else None,
            lens.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)) if lens is not None else None,
            _ptr(arr(h0), real) if h0 is not None else None,
            _ptr(arr(c0), real) if c0 is not None else None,
            _ptr(out, real), _ptr(h_n, real), _ptr(c_n, real))
    if rc != 0:
        raise RuntimeError(f"oracle_forward_{precision} failed with code {rc}")
    return out, h_n, c_n


def _sigmoid(v):
    return 1.0 / (1.0 + np.exp(-v))


def forward_numpy(x, w_ih, w_hh, b_ih, b_hh, w_lin, b_lin, *, lengths=None, h0=None, c0=None,
                  out_mode: str = "seq"):
    """Vectorised float64 restatement of reference.py:11-72 (same contract as `forward`)."""
    x = np.asarray(x, dtype=np.float64)
    B, T, _ = x.shape
    L = len(w_ih)
    H = np.asarray(w_hh[0]).shape[1]
    lens = np.full(B, T, dtype=np.int64) if lengths is None else np.clip(np.asarray(lengths), 0, T)
    layer_in = x
    h_n = np.zeros((L, B, H))
    c_n = np.zeros((L, B, H))
    for l in range(L):
        wi = np.asarray(w_ih[l], dtype=np.float64)
        wh = np.asarray(w_hh[l], dtype=np.float64)
        bias = np.zeros(4 * H)
        if b_ih is not None and b_ih[l] is not None:
            bias = bias + np.asarray(b_ih[l], dtype=np.float64)
        if b_hh is not None and b_hh[l] is not None:
            bias = bias + np.asarray(b_hh[l], dtype=np.float64)
        h = np.zeros((B, H)) if h0 is None else np.array(h0[l], dtype=np.float64)
        c = np.zeros((B, H)) if c0 is None else np.array(c0[l], dtype=np.float64)
        outs = np.zeros((B, T, H))
        for t in range(T):
            g = layer_in[:, t, :] @ wi.T + h @ wh.T + bias
            i, f, gg, o = np.split(g, 4, axis=1)
            c_new = _sigmoid(f) * c + _sigmoid(i) * np.tanh(gg)
            h_new = _sigmoid(o) * np.tanh(c_new)
            live = (t < lens)[:, None]
            c = np.where(live, c_new, c)
            h = np.where(live, h_new, h)
            outs[:, t, :] = np.where(live, h_new, 0.0)
        h_n[l] = h
        c_n[l] = c
        layer_in = outs
    if out_mode == "hseq":
        return layer_in, h_n, c_n
    w_lin = np.asarray(w_lin, dtype=np.float64)
    bl = np.zeros(w_lin.shape[0]) if b_lin is None else np.asarray(b_lin, dtype=np.float64)
    if out_mode == "last":
        idx = np.maximum(lens - 1, 0)
        last = layer_in[np.arange(B), idx, :]
        last = np.where((lens > 0)[:, None], last, h_n[L - 1])
        return last @ w_lin.T + bl, h_n, c_n
    out = layer_in @ w_lin.T + bl
    mask = (np.arange(T)[None, :] < lens[:, None])[:, :, None]
    return np.where(mask, out, 0.0), h_n, c_n


def unique_rows(x, *, lengths=None, h0=None, c0=None):
    """Groups identical batch rows: the general form of the reference's
    all-rows-equal check (persistent_lstm_hip/persistent_lstm_hip/model.py:
    493-520, ``torch.equal(x, x[:1].expand_as(x))``).

    A row's identity is the bytes of x[b, :len_b], len_b and, when given, the
    bytes of h0[:, b] and c0[:, b].  Returns (row_map[B], unique_index[U], U):
    distinct rows are numbered in order of first occurrence, unique_index
    lists each one's first row.
    """
    x = np.ascontiguousarray(x)
    B, T = x.shape[0], x.shape[1]
    lens = np.full(B, T, dtype=np.int64) if lengths is None else np.clip(np.asarray(lengths, dtype=np.int64), 0, T)
    seen = {}
    row_map = np.zeros(B, dtype=np.int32)
    first = []
    for b in range(B):
        key = (int(lens[b]), x[b, :lens[b]].tobytes())
        if h0 is not None:
            key += (np.ascontiguousarray(h0[:, b]).tobytes(), np.ascontiguousarray(c0[:, b]).tobytes())
        if key not in seen:
            seen[key] = len(first)
            first.append(b)
        row_map[b] = seen[key]
    return row_map, np.asarray(first, dtype=np.int32), len(first)
