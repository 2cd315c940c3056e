"""Two-GPU tests (skipped on a one-GPU box): the one-process multi-device driver
(shard.MultiDeviceRegressor, peer copies only) and the C ABI's promise to leave the
calling thread's current device as it found it."""
from __future__ import annotations

import ctypes

import pytest
import torch

from helpers import make_model, weights_of
import persistent_lstm_hip_b200 as plstm
from persistent_lstm_hip_b200 import _lib, core, shard

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def two_gpus():
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two CUDA devices")
    return [torch.device("cuda", 0), torch.device("cuda", 1)]


@pytest.mark.parametrize("varlen", [False, True])
def test_multi_device_regressor_equals_one_device(two_gpus, varlen):
    """Rows are independent, so the sharded forward equals the one-device forward bit for bit."""
    I, H, L, O, B, T = 5, 128, 4, 24, 300, 64
    native = make_model(I, H, L, O, seed=31).to(two_gpus[0]).half()
    model = plstm.convert_regressor_module(native)
    x = torch.randn(B, T, I, generator=torch.Generator().manual_seed(4)).to(two_gpus[0], torch.float16)
    lens = None
    if varlen:
        lens = torch.randint(1, T + 1, (B,), generator=torch.Generator().manual_seed(5), dtype=torch.int32)
    want = model(x, lengths=None if lens is None else lens.to(two_gpus[0]))
    seq_want, (h_want, c_want) = model.forward_sequence(x, lengths=None if lens is None else lens.to(two_gpus[0]))
    multi = shard.MultiDeviceRegressor(model, two_gpus)
    got = multi(x, lengths=lens)
    seq_got, (h_got, c_got) = multi.forward_sequence(x, lengths=lens)
    torch.cuda.synchronize(two_gpus[0])
    torch.cuda.synchronize(two_gpus[1])
    assert got.device == two_gpus[0]
    assert torch.equal(got, want)
    assert torch.equal(seq_got, seq_want)
    assert torch.equal(h_got, h_want) and torch.equal(c_got, c_want)


def test_entry_point_restores_the_current_device(two_gpus):
    """A C caller current on device 0 that runs a device-1 problem stays on device 0."""
    I, H, L, O = 5, 128, 4, 24
    w = weights_of(make_model(I, H, L, O, seed=32), L, torch.float16, two_gpus[1])
    pw = core.PackedWeights(*w, out_mode="last", backend="tc")
    x = torch.randn(8, 16, I, generator=torch.Generator().manual_seed(6)).to(two_gpus[1], torch.float16)
    out = torch.empty(8, O, dtype=torch.float16, device=two_gpus[1])
    d = pw.desc(batch=8, seq_len=16)
    nbytes = ctypes.c_size_t(0)
    lib = _lib.load()
    _lib.check(lib.plstm_workspace_size(ctypes.byref(d), ctypes.byref(nbytes)))
    ws = torch.empty(int(nbytes.value), dtype=torch.uint8, device=two_gpus[1])
    torch.cuda.set_device(two_gpus[0])
    s1 = torch.cuda.current_stream(two_gpus[1]).cuda_stream
    _lib.check(lib.plstm_forward_packed(ctypes.byref(d), pw.blob.data_ptr(), x.data_ptr(), None, None, None,
                                        out.data_ptr(), None, None, ws.data_ptr(), ws.numel(), s1))
    assert torch.cuda.current_device() == 0
    _lib.check(lib.plstm_forward_packed_noalloc(ctypes.byref(d), pw.blob.data_ptr(), x.data_ptr(), None, None,
                                                None, out.data_ptr(), None, None, s1))
    assert torch.cuda.current_device() == 0
    torch.cuda.synchronize(two_gpus[1])
    ref, _, _ = pw.forward(x, check=True, need_state=False)
    assert torch.equal(out, ref)
