"""The C-ABI library loads and exports every symbol include/plstm.h declares;
descriptor validation and error reporting work without a GPU."""
from __future__ import annotations

import ctypes
import os
import re

import pytest

from conftest import ROOT
from persistent_lstm_hip_b200 import _lib


def declared_symbols():
    names = set()
    for fn in os.listdir(os.path.join(ROOT, "include")):
        if fn.endswith(".h"):
            text = open(os.path.join(ROOT, "include", fn)).read()
            names.update(re.findall(r"PLSTM_API\s+[\w\s\*]+?\b(plstm_\w+)\s*\(", text))
    return sorted(names)


def test_header_declares_entry_points():
    names = declared_symbols()
    assert "plstm_forward" in names and "plstm_persistent_lstm4_forward_interleaved" in names
    assert len(names) >= 19


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    for name in declared_symbols():
        assert hasattr(lib, name), f"libplstm.so does not export {name}"
        assert name in _lib.PROTOTYPES, f"_lib.PROTOTYPES lacks {name}"


def test_abi_version():
    assert _lib.load().plstm_abi_version() == 1


def _desc(**kw):
    base = dict(batch=4, seq_len=3, input_size=5, hidden_size=16, num_layers=2, output_size=3,
                dtype=_lib.F32, w_layout=0, flags=_lib.FLAG_OUT_SEQ, backend=0, timeout_ms=0, device=0)
    base.update(kw)
    return _lib.Desc(*[base[f] for f, _ in _lib.Desc._fields_])


@pytest.mark.parametrize("bad, msg", [
    (dict(batch=-1), "batch"),
    (dict(hidden_size=0), "hidden_size"),
    (dict(num_layers=0), "num_layers"),
    (dict(dtype=7), "dtype"),
    (dict(flags=_lib.FLAG_OUT_SEQ | _lib.FLAG_OUT_LAST), "exactly one"),
    (dict(flags=0), "exactly one"),
    (dict(output_size=0), "output_size"),
    (dict(w_layout=9), "w_layout"),
])
def test_descriptor_validation(bad, msg):
    lib = _lib.load()
    n = ctypes.c_size_t(0)
    rc = lib.plstm_workspace_size(ctypes.byref(_desc(**bad)), ctypes.byref(n))
    assert rc == _lib.EINVAL
    assert msg in _lib.last_error()


def test_sizes_are_positive_and_scale():
    lib = _lib.load()
    small, big = ctypes.c_size_t(0), ctypes.c_size_t(0)
    assert lib.plstm_workspace_size(ctypes.byref(_desc(batch=4)), ctypes.byref(small)) == 0
    assert lib.plstm_workspace_size(ctypes.byref(_desc(batch=64)), ctypes.byref(big)) == 0
    assert 0 < small.value < big.value
    pk = ctypes.c_size_t(0)
    assert lib.plstm_packed_size(ctypes.byref(_desc()), ctypes.byref(pk)) == 0 and pk.value > 0


def test_forward_rejects_null_and_small_workspace():
    lib = _lib.load()
    d = _desc()
    rc = lib.plstm_forward_packed(ctypes.byref(d), None, None, None, None, None, None, None, None, None, 0, None)
    assert rc == _lib.EINVAL and "packed" in _lib.last_error()
    rc = lib.plstm_forward_packed(ctypes.byref(d), 16, 16, None, None, None, 16, None, None, 16, 8, None)
    assert rc == _lib.EWORKSPACE


def test_forward_rejects_unaligned_buffers():
    # Packed images and workspaces are read with 16-byte vector loads and bulk copies; a
    # misaligned pointer is refused on the host before any launch (no pointer is dereferenced).
    lib = _lib.load()
    d = _desc()
    for packed, ws in ((24, 16), (16, 8), (1040, 1028)):
        rc = lib.plstm_forward_packed(ctypes.byref(d), packed, 16, None, None, None, 16, None, None, ws, 1 << 30,
                                      None)
        assert rc == _lib.EINVAL and "16-byte aligned" in _lib.last_error()
    ptrs = (ctypes.c_void_p * 2)(16, 16)
    rc = lib.plstm_pack(ctypes.byref(d), ptrs, ptrs, None, None, 16, None, 24, 1 << 30, None)
    assert rc == _lib.EINVAL and "16-byte aligned" in _lib.last_error()


def test_tc_backend_refused_without_b200():
    # Forcing the tensor-core backend on a host without an sm_100 device is ENOTSUP, not a fallback.
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    lib = _lib.load()
    d = _desc(dtype=_lib.F16, hidden_size=128, num_layers=4, backend=_lib.BACKEND_TC)
    n = ctypes.c_size_t(0)
    assert lib.plstm_workspace_size(ctypes.byref(d), ctypes.byref(n)) == _lib.ENOTSUP
    assert "tensor-core backend cannot serve" in _lib.last_error()
