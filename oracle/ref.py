"""ctypes binding of oracle/_ref/libplstm_ref.so, the reference's own CPU implementation
of the fixed 4-layer LSTM + Linear path (persistent_lstm4_forward_reference,
persistent_lstm_hip/csrc/persistent_lstm_reference.cpp:42-64), built by build_ref.py.

Test and benchmark infrastructure only (the parity checker and the timed CPU
baseline); the product never imports it.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "_ref", "libplstm_ref.so")
_lib = None


def available() -> bool:
    return os.path.exists(LIB)


def _load():
    global _lib
    if _lib is None:
        import torch  # noqa: F401  (loads libtorch into the process before the shim)

        lib = ctypes.CDLL(LIB)
        P, I32 = ctypes.c_void_p, ctypes.c_int
        PP = ctypes.POINTER(ctypes.c_void_p)
        lib.plstm_ref4_forward.restype = I32
        lib.plstm_ref4_forward.argtypes = [I32, P, I32, I32, I32, I32, I32, PP, PP, PP, P, P, P, I32]
        _lib = lib
    return _lib


def forward(x, w_ih, w_hh, b_ih, b_hh, w_lin, b_lin, *, precision: str = "f64", threads: int = 0) -> np.ndarray:
    """out[B, O] of the reference's CPU path for x[B, T, I] and 4 layers of nn.LSTM weights
    (the reference takes the pre-summed bias b_ih + b_hh, as its Python wrapper passes it)."""
    if len(w_ih) != 4:
        raise ValueError("the reference's CPU path is the fixed 4-layer model")
    dt = np.float64 if precision == "f64" else np.float32
    c = lambda a: np.ascontiguousarray(a, dtype=dt)
    x = c(x)
    B, T, I = x.shape
    H = int(np.asarray(w_hh[0]).shape[1])
    O = int(np.asarray(w_lin).shape[0])
    keep = [c(w) for w in w_ih] + [c(w) for w in w_hh] + [c(np.asarray(bi) + np.asarray(bh)) for bi, bh in zip(b_ih, b_hh)]
    arr = lambda ts: (ctypes.c_void_p * 4)(*[t.ctypes.data for t in ts])
    a_ih, a_hh, a_b = arr(keep[0:4]), arr(keep[4:8]), arr(keep[8:12])
    wl, bl = c(w_lin), c(b_lin)
    out = np.empty((B, O), dtype=dt)
    PP = ctypes.POINTER(ctypes.c_void_p)
    rc = _load().plstm_ref4_forward(1 if dt == np.float64 else 0, x.ctypes.data, B, T, I, H, O,
                                    ctypes.cast(a_ih, PP), ctypes.cast(a_hh, PP), ctypes.cast(a_b, PP),
                                    wl.ctypes.data, bl.ctypes.data, out.ctypes.data, int(threads))
    if rc != 0:
        raise RuntimeError("persistent_lstm4_forward_reference raised a C++ exception")
    return out
