"""tcgen05 input-projection GEMM vs a plain PyTorch f32 matmul of the same 16-bit inputs."""
from __future__ import annotations

import pytest
import torch

from persistent_lstm_hip_b200.adaptive_ext import adaptive_lstm_input_gemm_forward_workspace

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M, K, N", [(1000, 5, 512), (128, 16, 64), (777, 128, 512), (300, 256, 1024),
                                     (129, 8, 136), (5000, 5, 1024), (1, 64, 2048)])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_input_gemm_matches_torch_f32(cuda_device, M, K, N, dtype):
    g = torch.Generator().manual_seed(M + K + N)
    x = torch.randn(M, K, generator=g).to(cuda_device, dtype)
    w_t = (torch.rand(K, N, generator=g) * 0.2 - 0.1).to(cuda_device, dtype)
    gate = torch.full((M, N), float("nan"), device=cuda_device, dtype=dtype)
    out = adaptive_lstm_input_gemm_forward_workspace(x, w_t, gate)
    assert out.data_ptr() == gate.data_ptr()
    ref = x.float() @ w_t.float()
    # The kernel accumulates in f32 and rounds once to the 16-bit type: within half a unit in the
    # last place of it (2^-11 relative for f16, 2^-8 for bf16), with a factor of 2 for the f32
    # summation order; a dropped or doubled K step would exceed it.
    rtol = 2.0 ** -10 if dtype == torch.float16 else 2.0 ** -7
    torch.testing.assert_close(gate.float(), ref, rtol=rtol, atol=1e-5)


def test_input_gemm_rejects_bad_args(cuda_device):
    x = torch.zeros(4, 5, device=cuda_device, dtype=torch.float16)
    w = torch.zeros(6, 8, device=cuda_device, dtype=torch.float16)
    with pytest.raises(ValueError):
        adaptive_lstm_input_gemm_forward_workspace(x, w, torch.zeros(4, 8, device=cuda_device, dtype=torch.float16))
