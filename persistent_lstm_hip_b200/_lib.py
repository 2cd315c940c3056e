"""ctypes binding of the in-tree CUDA library (lib/libplstm.so, include/plstm.h).

The library is the product path: there is no CPU or PyTorch fallback.  If it
cannot be loaded, every entry point raises ``PlstmUnavailable``.
"""
from __future__ import annotations

import ctypes
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.environ.get("PLSTM_LIB", os.path.join(HERE, "lib", "libplstm.so"))

OK, EINVAL, ENOTSUP, ETIMEOUT, ECUDA, EWORKSPACE, EBOUNDS = 0, 1, 2, 3, 4, 5, 6
F32, F16, BF16 = 0, 1, 2
W_NATIVE, W_TRANSPOSED, W_KPAIR, W_MMAC = 0, 1, 2, 3
HU_SEQ_MAJOR, HU_WRITE_SEQUENCE = 0x1, 0x2
BACKEND_AUTO, BACKEND_SIMT, BACKEND_TC = 0, 1, 2
FLAG_OUT_SEQ = 0x1
FLAG_OUT_LAST = 0x2
FLAG_NO_LINEAR = 0x4
FLAG_BIAS_SUMMED = 0x8
FLAG_SYNC_CHECK = 0x10
FLAG_CN_F32 = 0x20
FLAG_DEDUPE = 0x40
FLAG_TEST_DROP = 0x100
FLAG_TRACE = 0x200

_CODE_NAMES = {EINVAL: "PLSTM_EINVAL", ENOTSUP: "PLSTM_ENOTSUP", ETIMEOUT: "PLSTM_ETIMEOUT",
               ECUDA: "PLSTM_ECUDA", EWORKSPACE: "PLSTM_EWORKSPACE", EBOUNDS: "PLSTM_EBOUNDS"}

# Every symbol include/plstm.h declares, with its ctypes prototype.
_P = ctypes.c_void_p
_I32 = ctypes.c_int32
_SZ = ctypes.c_size_t
_PP = ctypes.POINTER(ctypes.c_void_p)


class Desc(ctypes.Structure):
    """plstm_desc."""
    _fields_ = [(n, ctypes.c_int32) for n in (
        "batch", "seq_len", "input_size", "hidden_size", "num_layers", "output_size", "dtype",
        "w_layout", "flags", "backend", "timeout_ms", "device")]


_DP = ctypes.POINTER(Desc)
PROTOTYPES = {
    "plstm_abi_version": (_I32, []),
    "plstm_last_error": (ctypes.c_char_p, []),
    "plstm_select_backend": (_I32, [_DP]),
    "plstm_packed_size": (_I32, [_DP, ctypes.POINTER(_SZ)]),
    "plstm_pack": (_I32, [_DP, _PP, _PP, _PP, _PP, _P, _P, _P, _SZ, _P]),
    "plstm_workspace_size": (_I32, [_DP, ctypes.POINTER(_SZ)]),
    "plstm_forward_packed": (_I32, [_DP, _P, _P, _P, _P, _P, _P, _P, _P, _P, _SZ, _P]),
    "plstm_forward": (_I32, [_DP, _P, _PP, _PP, _PP, _PP, _P, _P, _P, _P, _P, _P, _P, _P, _P, _SZ, _P]),
    "plstm_unique_rows_workspace_size": (_I32, [_DP, ctypes.POINTER(_SZ)]),
    "plstm_unique_rows": (_I32, [_DP, _P, _P, _P, _P, _P, _P, ctypes.POINTER(_I32), _P, _SZ, _P]),
    "plstm_read_status": (_I32, [_P, _P, ctypes.POINTER(_I32), ctypes.POINTER(_I32)]),
    "plstm_forward_packed_noalloc": (_I32, [_DP, _P, _P, _P, _P, _P, _P, _P, _P, _P]),
    "plstm_ref4_workspace_size": (_I32, [_I32, _I32, _I32, _I32, _I32, ctypes.POINTER(_SZ)]),
    "plstm_persistent_lstm4_forward": (_I32, [_P, _I32, _I32, _I32, _I32, _I32, _PP, _PP, _PP, _P, _P, _P, _P, _SZ, _P]),
    "plstm_persistent_lstm4_forward_packed": (_I32, [_P, _I32, _I32, _I32, _I32, _I32, _PP, _PP, _PP, _P, _P, _P, _P, _SZ, _P]),
    "plstm_persistent_lstm4_forward_interleaved": (_I32, [_P, _I32, _I32, _I32, _I32, _I32, _PP, _PP, _PP, _P, _P, _P, _P, _SZ, _P]),
    "plstm_persistent_lstm4_forward_monolithic": (_I32, [_P, _I32, _I32, _I32, _I32, _I32, _PP, _PP, _PP, _P, _P, _P, _P, _SZ, _P]),
    "plstm_persistent_lstm4_forward_projected": (_I32, [_P, _I32, _I32, _I32, _I32, _I32, _PP, _PP, _PP, _P, _P, _P, _P, _SZ, _P]),
    "plstm_regressor_forward_generic": (_I32, [_P, _I32, _I32, _I32, _I32, _I32, _I32, _PP, _PP, _PP, _P, _P, _P, _P, _SZ, _P]),
    "plstm_repeat_first_row": (_I32, [_P, _I32, _I32, _I32, _P, _P]),
    "plstm_input_gemm": (_I32, [_P, _I32, _I32, _P, _I32, _I32, _P, _P]),
    "plstm_hidden_update_workspace_size": (_I32, [_I32, _I32, _I32, _I32, _I32, _I32, ctypes.POINTER(_SZ)]),
    "plstm_hidden_update": (_I32, [_P, _I32, _I32, _I32, _P, _I32, _P, _I32, _I32, _P, _P, _P, _P, _SZ, _P]),
    "plstm_diag_tmem_layout": (_I32, [_P, _P]),
    "plstm_diag_step_latency": (_I32, [_I32, _I32, _I32, _P, _I32, _P]),
    "plstm_launch_count": (ctypes.c_int64, []),
    "plstm_profile": (_I32, [_I32]),
    "plstm_profile_read": (_I32, [ctypes.POINTER(ctypes.c_float), ctypes.POINTER(_I32)]),
}


class PlstmError(RuntimeError):
    """A C-ABI call returned a PLSTM_E* code."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"{_CODE_NAMES.get(code, code)}: {msg}")
        self.code = code


class PlstmUnavailable(ImportError):
    """The CUDA library is missing or cannot be loaded (no fallback exists)."""


_lock = threading.Lock()
_lib = None


def load():
    """Loads lib/libplstm.so once; raises PlstmUnavailable if it cannot."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise PlstmUnavailable(
                    f"{LIB_PATH} is missing: build it with `python -m persistent_lstm_hip_b200.build` "
                    "(there is no CPU fallback)")
            try:
                lib = ctypes.CDLL(LIB_PATH)
            except OSError as exc:
                raise PlstmUnavailable(f"cannot load {LIB_PATH}: {exc}") from exc
            for name, (res, args) in PROTOTYPES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def last_error() -> str:
    return (load().plstm_last_error() or b"").decode(errors="replace")


def check(rc: int) -> None:
    if rc != OK:
        raise PlstmError(rc, last_error())


def ptr_array(ptrs):
    """A C array of void* (None -> NULL) for the `const void* const*` arguments."""
    arr = (ctypes.c_void_p * len(ptrs))(*[p if p else None for p in ptrs])
    return ctypes.cast(arr, _PP), arr
