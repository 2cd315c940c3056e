"""Torch-facing functional API over the C ABI.

PyTorch only provides device memory (through its caching allocator) and the
current CUDA stream here; all computation happens in lib/libplstm.so.

* ``PackedWeights``: the device image of an LSTM stack + Linear head in the
  layout the selected backend reads (``plstm_pack``).  It replaces the
  per-weight-version caches of the reference's Python wrappers
  (persistent_lstm_hip/persistent_lstm_hip/model.py:542-582,
  miopen_adaptive_lstm_hip/miopen_adaptive_lstm_hip/model.py:403-430).
* ``lstm_linear_forward``: x[B,T,I] + per-layer weights + Linear head ->
  (out, h_n, c_n), the north-star entry point.
"""
from __future__ import annotations

import ctypes
import collections
import os
import threading
from typing import Optional, Sequence, Tuple

import torch

from . import _lib

_DTYPES = {torch.float32: _lib.F32, torch.float16: _lib.F16, torch.bfloat16: _lib.BF16}
_BACKENDS = {"auto": _lib.BACKEND_AUTO, "simt": _lib.BACKEND_SIMT, "tc": _lib.BACKEND_TC}
_OUT_FLAGS = {"seq": _lib.FLAG_OUT_SEQ, "last": _lib.FLAG_OUT_LAST, "hseq": _lib.FLAG_NO_LINEAR}


def _env_check() -> bool:
    return os.environ.get("PLSTM_SYNC_CHECK", "0") not in ("", "0", "false", "off")


def _ptr(t: Optional[torch.Tensor]):
    return None if t is None else t.data_ptr()


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _require_cuda(t: torch.Tensor, name: str, device: torch.device, dtype=None) -> torch.Tensor:
    if not isinstance(t, torch.Tensor):
        raise TypeError(f"{name} must be a torch.Tensor")
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (this path has no CPU implementation)")
    if t.device != device:
        raise ValueError(f"{name} is on {t.device}, expected {device}")
    if dtype is not None and t.dtype != dtype:
        raise ValueError(f"{name} has dtype {t.dtype}, expected {dtype}")
    return t.contiguous()


class DeviceStatus:
    """Reports device-side failures of forwards that ran without a synchronising check.

    The kernels record a bounded inter-CTA wait that gave up (PLSTM_ETIMEOUT and
    the failing CTA / step) in the status word at the start of the call's
    workspace.  Without PLSTM_FLAG_SYNC_CHECK nothing reads that word before the
    temporary workspace is freed, so after every such forward the word is copied
    asynchronously into pinned host memory, on the same stream, behind an event.
    The next forward on the device (or ``check_device_status``) looks at every
    copy whose event has completed, without synchronising, and raises
    ``PlstmError(PLSTM_ETIMEOUT)`` for the first failure it finds.  Forwards
    captured into a CUDA graph are not watched (read their status with
    ``plstm_read_status`` on a workspace the caller keeps).
    """

    RING = 64  # copies in flight per device before the oldest one is waited for

    def __init__(self, device: torch.device):
        self.device = device
        self.host = torch.zeros(self.RING, 2, dtype=torch.int32, pin_memory=True)
        self.events = [None] * self.RING
        self.pending = collections.deque()
        self.next = 0
        self.lock = threading.Lock()

    def _retire(self, wait: bool) -> None:
        while self.pending:
            slot = self.pending[0]
            ev = self.events[slot]
            if not wait and not ev.query():
                return
            ev.synchronize()
            self.pending.popleft()
            self.events[slot] = None
            st, detail = (int(v) for v in self.host[slot].tolist())
            if st != _lib.OK:
                raise _lib.PlstmError(
                    st, f"device status {st} (cta {detail >> 16}, step {detail & 0xffff}) of an earlier forward "
                        f"on {self.device}: a bounded inter-CTA wait gave up; its outputs are incomplete")

    def poll(self, wait: bool = False) -> None:
        """Raises for a failed earlier forward whose status copy has landed (all of them with wait=True).
        Does nothing while the current stream is being captured into a CUDA graph (event queries
        are not allowed then)."""
        if torch.cuda.is_current_stream_capturing():
            return
        with self.lock:
            self._retire(wait)

    def watch(self, ws: torch.Tensor, stream: torch.cuda.Stream) -> None:
        """Enqueues the status copy of the forward just enqueued on `stream` with workspace `ws`.
        Forwards captured into a CUDA graph are not watched."""
        if torch.cuda.is_current_stream_capturing():
            return
        with self.lock:
            while len(self.pending) >= self.RING:  # only when the host runs 64 forwards ahead of the GPU
                self._retire(True)
            slot = self.next
            self.next = (slot + 1) % self.RING
            with torch.cuda.stream(stream):
                self.host[slot].copy_(ws[:8].view(torch.int32), non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(stream)
            self.events[slot] = ev
            self.pending.append(slot)


_status_lock = threading.Lock()
_status = {}


def device_status(device: torch.device) -> DeviceStatus:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    with _status_lock:
        st = _status.get(idx)
        if st is None:
            st = _status[idx] = DeviceStatus(torch.device("cuda", idx))
        return st


def check_device_status(device: Optional[torch.device] = None) -> None:
    """Waits for the status copies of every unchecked forward on `device` (default: the
    current device) and raises PlstmError(PLSTM_ETIMEOUT) if one of them failed."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    device_status(dev).poll(wait=True)


def make_desc(*, batch: int, seq_len: int, input_size: int, hidden_size: int, num_layers: int,
              output_size: int, dtype: torch.dtype, flags: int, backend: str = "auto",
              w_layout: int = _lib.W_NATIVE, timeout_ms: int = 0, device: int = 0) -> _lib.Desc:
    if dtype not in _DTYPES:
        raise ValueError(f"unsupported dtype {dtype}; use float32, float16 or bfloat16")
    if backend not in _BACKENDS:
        raise ValueError(f"backend must be one of {sorted(_BACKENDS)}")
    return _lib.Desc(batch, seq_len, input_size, hidden_size, num_layers, output_size, _DTYPES[dtype],
                     w_layout, flags, _BACKENDS[backend], timeout_ms, device)


def select_backend(*, input_size: int, hidden_size: int, num_layers: int, output_size: int,
                   dtype: torch.dtype, out_mode: str = "seq", backend: str = "auto",
                   device: int = 0) -> str:
    """Name of the backend ("tc" or "simt") plstm_forward would run."""
    d = make_desc(batch=1, seq_len=1, input_size=input_size, hidden_size=hidden_size,
                  num_layers=num_layers, output_size=output_size, dtype=dtype,
                  flags=_OUT_FLAGS[out_mode], backend=backend, device=device)
    b = _lib.load().plstm_select_backend(ctypes.byref(d))
    if b < 0:
        _lib.check(-b)
    return {_lib.BACKEND_SIMT: "simt", _lib.BACKEND_TC: "tc"}[b]


class PackedWeights:
    """Device image of the weights for one (shape, dtype, output mode, backend)."""

    def __init__(self, w_ih: Sequence[torch.Tensor], w_hh: Sequence[torch.Tensor],
                 b_ih: Optional[Sequence[Optional[torch.Tensor]]], b_hh: Optional[Sequence[Optional[torch.Tensor]]],
                 w_lin: Optional[torch.Tensor], b_lin: Optional[torch.Tensor], *, out_mode: str = "seq",
                 backend: str = "auto", w_layout: int = _lib.W_NATIVE, input_size: Optional[int] = None,
                 hidden_size: Optional[int] = None):
        if out_mode not in _OUT_FLAGS:
            raise ValueError(f"out_mode must be one of {sorted(_OUT_FLAGS)}")
        if len(w_ih) == 0 or len(w_ih) != len(w_hh):
            raise ValueError("w_ih and w_hh must be non-empty lists of the same length")
        lib = _lib.load()
        dev = w_ih[0].device
        dtype = w_ih[0].dtype
        L = len(w_ih)
        if hidden_size is None:
            if w_layout != _lib.W_NATIVE:
                raise ValueError("hidden_size is required for non-native weight layouts")
            hidden_size = int(w_hh[0].shape[1])
        if input_size is None:
            if w_layout != _lib.W_NATIVE:
                raise ValueError("input_size is required for non-native weight layouts")
            input_size = int(w_ih[0].shape[1])
        H = hidden_size
        if w_layout == _lib.W_NATIVE:
            for l in range(L):
                k = input_size if l == 0 else H
                if tuple(w_ih[l].shape) != (4 * H, k):
                    raise ValueError(f"w_ih[{l}] must be [{4 * H}, {k}], got {tuple(w_ih[l].shape)}")
                if tuple(w_hh[l].shape) != (4 * H, H):
                    raise ValueError(f"w_hh[{l}] must be [{4 * H}, {H}], got {tuple(w_hh[l].shape)}")
        O = 0
        if out_mode != "hseq":
            if w_lin is None:
                raise ValueError("w_lin is required unless out_mode='hseq'")
            if w_lin.dim() != 2 or w_lin.shape[1] != H:
                raise ValueError(f"w_lin must be [O, {H}], got {tuple(w_lin.shape)}")
            O = int(w_lin.shape[0])
        keep = []

        def conv(t, name):
            if t is None:
                return None
            t = _require_cuda(t, name, dev, dtype)
            keep.append(t)
            return t

        w_ih = [conv(t, f"w_ih[{i}]") for i, t in enumerate(w_ih)]
        w_hh = [conv(t, f"w_hh[{i}]") for i, t in enumerate(w_hh)]
        flags = _OUT_FLAGS[out_mode]
        if b_ih is not None:
            b_ih = [conv(t, f"b_ih[{i}]") for i, t in enumerate(b_ih)]
        if b_hh is not None:
            b_hh = [conv(t, f"b_hh[{i}]") for i, t in enumerate(b_hh)]
        elif b_ih is not None:
            flags |= _lib.FLAG_BIAS_SUMMED
        w_lin = conv(w_lin, "w_lin") if out_mode != "hseq" else None
        b_lin = conv(b_lin, "b_lin") if out_mode != "hseq" else None
        self.device = dev
        self.dtype = dtype
        self.input_size, self.hidden_size, self.num_layers, self.output_size = input_size, H, L, O
        self.out_mode = out_mode
        self.backend_request = backend
        self._flags = flags
        d = self.desc(batch=1, seq_len=1)
        d.w_layout = w_layout
        nbytes = ctypes.c_size_t(0)
        with torch.cuda.device(dev):
            _lib.check(lib.plstm_packed_size(ctypes.byref(d), ctypes.byref(nbytes)))
            self.blob = torch.empty(int(nbytes.value), dtype=torch.uint8, device=dev)
            a_ih, _k1 = _lib.ptr_array([_ptr(t) for t in w_ih])
            a_hh, _k2 = _lib.ptr_array([_ptr(t) for t in w_hh])
            a_bih = _lib.ptr_array([_ptr(t) for t in b_ih])[0] if b_ih is not None else None
            a_bhh = _lib.ptr_array([_ptr(t) for t in b_hh])[0] if b_hh is not None else None
            keep.append((_k1, _k2, a_bih, a_bhh))
            _lib.check(lib.plstm_pack(ctypes.byref(d), a_ih, a_hh, a_bih, a_bhh, _ptr(w_lin), _ptr(b_lin),
                                      self.blob.data_ptr(), self.blob.numel(), _stream(dev)))
        # The pack kernels read the source tensors asynchronously on the current stream.
        for t in keep:
            if isinstance(t, torch.Tensor):
                t.record_stream(torch.cuda.current_stream(dev))
        self.backend = select_backend(input_size=input_size, hidden_size=H, num_layers=L, output_size=max(O, 1),
                                      dtype=dtype, out_mode=out_mode, backend=backend, device=dev.index)

    def desc(self, *, batch: int, seq_len: int, extra_flags: int = 0, timeout_ms: int = 0) -> _lib.Desc:
        return make_desc(batch=batch, seq_len=seq_len, input_size=self.input_size, hidden_size=self.hidden_size,
                         num_layers=self.num_layers, output_size=max(self.output_size, 1), dtype=self.dtype,
                         flags=self._flags | extra_flags, backend=self.backend_request, timeout_ms=timeout_ms,
                         device=self.device.index or 0)

    def forward(self, x: torch.Tensor, *, lengths: Optional[torch.Tensor] = None,
                hx: Optional[Tuple[torch.Tensor, torch.Tensor]] = None, need_state: bool = True,
                check: Optional[bool] = None, timeout_ms: int = 0, extra_flags: int = 0,
                c_n_f32: bool = False, dedupe: bool = False):
        """Runs the LSTM + Linear forward on x[B,T,I]; returns (out, h_n, c_n).

        dedupe=True computes each distinct row (x up to its length, the length,
        its hx rows) once and copies the results to the duplicates
        (PLSTM_FLAG_DEDUPE); it synchronises the stream once.
        """
        lib = _lib.load()
        dev = self.device
        x = _require_cuda(x, "x", dev, self.dtype)
        if x.dim() != 3 or x.shape[2] != self.input_size:
            raise ValueError(f"x must be [B, T, {self.input_size}], got {tuple(x.shape)}")
        B, T, _ = (int(v) for v in x.shape)
        L, H, O = self.num_layers, self.hidden_size, self.output_size
        lens = None
        if lengths is not None:
            lens = lengths.to(device=dev, dtype=torch.int32).contiguous()
            if lens.shape != (B,):
                raise ValueError(f"lengths must be [{B}], got {tuple(lens.shape)}")
        h0 = c0 = None
        if hx is not None:
            h0 = _require_cuda(hx[0], "h0", dev, self.dtype)
            c0 = _require_cuda(hx[1], "c0", dev, self.dtype)
            if tuple(h0.shape) != (L, B, H) or tuple(c0.shape) != (L, B, H):
                raise ValueError(f"hx tensors must be [{L}, {B}, {H}]")
        if self.out_mode == "seq":
            out = torch.empty(B, T, O, dtype=self.dtype, device=dev)
        elif self.out_mode == "last":
            out = torch.empty(B, O, dtype=self.dtype, device=dev)
        else:
            out = torch.empty(B, T, H, dtype=self.dtype, device=dev)
        h_n = c_n = None
        if need_state:
            h_n = torch.empty(L, B, H, dtype=self.dtype, device=dev)
            c_n = torch.empty(L, B, H, dtype=torch.float32 if c_n_f32 else self.dtype, device=dev)
        flags = extra_flags | (_lib.FLAG_CN_F32 if c_n_f32 else 0) | (_lib.FLAG_DEDUPE if dedupe else 0)
        sync_check = check if check is not None else _env_check()
        if sync_check:
            flags |= _lib.FLAG_SYNC_CHECK
        watcher = device_status(dev)
        watcher.poll()  # a failure of an earlier unchecked forward surfaces here
        d = self.desc(batch=B, seq_len=T, extra_flags=flags, timeout_ms=timeout_ms)
        nbytes = ctypes.c_size_t(0)
        _lib.check(lib.plstm_workspace_size(ctypes.byref(d), ctypes.byref(nbytes)))
        ws = torch.empty(max(int(nbytes.value), 256), dtype=torch.uint8, device=dev)
        with torch.cuda.device(dev):
            rc = lib.plstm_forward_packed(ctypes.byref(d), self.blob.data_ptr(), _ptr(x), _ptr(lens), _ptr(h0),
                                          _ptr(c0), _ptr(out), _ptr(h_n), _ptr(c_n), ws.data_ptr(), ws.numel(),
                                          _stream(dev))
        _lib.check(rc)
        if not sync_check:
            watcher.watch(ws, torch.cuda.current_stream(dev))
        return out, h_n, c_n


def lstm_linear_forward(x: torch.Tensor, w_ih: Sequence[torch.Tensor], w_hh: Sequence[torch.Tensor],
                        b_ih: Optional[Sequence[torch.Tensor]], b_hh: Optional[Sequence[torch.Tensor]],
                        w_lin: Optional[torch.Tensor] = None, b_lin: Optional[torch.Tensor] = None, *,
                        lengths: Optional[torch.Tensor] = None,
                        hx: Optional[Tuple[torch.Tensor, torch.Tensor]] = None, out_mode: str = "seq",
                        backend: str = "auto", check: Optional[bool] = None, dedupe: bool = False):
    """x[B,T,I] with nn.LSTM(batch_first=True)-layout weights -> (out, h_n, c_n).

    out is [B,T,O] for out_mode="seq" (zero past each row's length), [B,O] for
    "last" (Linear on each row's last valid step) and the last layer's h
    sequence [B,T,H] for "hseq".  h_n / c_n are [L,B,H] at each row's last
    valid step.  dedupe=True computes identical rows once (PLSTM_FLAG_DEDUPE).
    """
    packed = PackedWeights(w_ih, w_hh, b_ih, b_hh, w_lin, b_lin, out_mode=out_mode, backend=backend,
                           input_size=int(x.shape[-1]))
    return packed.forward(x, lengths=lengths, hx=hx, check=check, dedupe=dedupe)


def unique_rows(x: torch.Tensor, *, lengths: Optional[torch.Tensor] = None,
                hx: Optional[Tuple[torch.Tensor, torch.Tensor]] = None, hidden_size: Optional[int] = None,
                num_layers: Optional[int] = None) -> Tuple[torch.Tensor, torch.Tensor, int]:
    """Groups the identical rows of x[B,T,I] on the GPU (plstm_unique_rows).

    A row's identity is x up to its length, the length and, with hx, its h0 /
    c0 rows in every layer, compared bit for bit.  Returns (row_map[B],
    unique_index[count], count): row_map[b] is the distinct-row index of row
    b, unique_index the first row of each distinct row, ascending.  This is
    the general form of the reference's all-rows-equal check
    (persistent_lstm_hip/model.py:493-520).
    """
    lib = _lib.load()
    if not isinstance(x, torch.Tensor) or x.dim() != 3:
        raise ValueError("x must be a [B, T, I] tensor")
    dev = x.device
    x = _require_cuda(x, "x", dev)
    if x.dtype not in _DTYPES:
        raise ValueError(f"unsupported dtype {x.dtype}")
    B, T, I = (int(v) for v in x.shape)
    lens = None
    if lengths is not None:
        lens = lengths.to(device=dev, dtype=torch.int32).contiguous()
        if lens.shape != (B,):
            raise ValueError(f"lengths must be [{B}], got {tuple(lens.shape)}")
    h0 = c0 = None
    H, L = hidden_size or 1, num_layers or 1
    if hx is not None:
        h0 = _require_cuda(hx[0], "h0", dev, x.dtype)
        c0 = _require_cuda(hx[1], "c0", dev, x.dtype)
        if h0.dim() != 3 or h0.shape != c0.shape or int(h0.shape[1]) != B:
            raise ValueError(f"hx tensors must both be [L, {B}, H]")
        L, H = int(h0.shape[0]), int(h0.shape[2])
    d = make_desc(batch=B, seq_len=T, input_size=I, hidden_size=H, num_layers=L, output_size=1, dtype=x.dtype,
                  flags=_lib.FLAG_OUT_LAST, device=dev.index or 0)
    nbytes = ctypes.c_size_t(0)
    _lib.check(lib.plstm_unique_rows_workspace_size(ctypes.byref(d), ctypes.byref(nbytes)))
    ws = torch.empty(max(int(nbytes.value), 256), dtype=torch.uint8, device=dev)
    row_map = torch.empty(B, dtype=torch.int32, device=dev)
    uniq = torch.empty(B, dtype=torch.int32, device=dev)
    count = ctypes.c_int32(0)
    with torch.cuda.device(dev):
        rc = lib.plstm_unique_rows(ctypes.byref(d), _ptr(x), _ptr(lens), _ptr(h0), _ptr(c0), row_map.data_ptr(),
                                   uniq.data_ptr(), ctypes.byref(count), ws.data_ptr(), ws.numel(), _stream(dev))
    _lib.check(rc)
    return row_map, uniq[:count.value], int(count.value)


def read_status(ws: torch.Tensor) -> Tuple[int, int]:
    lib = _lib.load()
    st = ctypes.c_int32(0)
    detail = ctypes.c_int32(0)
    _lib.check(lib.plstm_read_status(ws.data_ptr(), _stream(ws.device), ctypes.byref(st), ctypes.byref(detail)))
    return st.value, detail.value
