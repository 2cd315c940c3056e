"""Host-side pieces of the hidden-update entry point: the MMAC-packed weight index
(PLSTM_W_MMAC, include/plstm.h) restated here is pinned bit-exactly against the
reference's own `_pack_mmac_weight` output (tests/golden/ref_mmac_h32.npz), and the
adaptive package mirror exposes every function of the reference's `_C` extension."""
from __future__ import annotations

import numpy as np

from conftest import load_golden
import persistent_lstm_hip_b200 as plstm


def mmac_index(H: int, r: int, k: int) -> int:
    """Element (r, k) of a [4H][H] recurrent weight in the MMAC-packed layout:
    [H/16 unit tiles][H/16 k tiles][16 k][4 unit groups][4 gates][4 units]."""
    gate, u = divmod(r, H)
    nt = H // 16
    return (((((u >> 4) * nt + (k >> 4)) * 16 + (k & 15)) * 4 + ((u & 15) >> 2)) * 4 + gate) * 4 + (u & 3)


def test_mmac_layout_matches_reference_packer():
    g = load_golden("ref_mmac_h32")
    w, packed = g["weight"], g["packed"]
    H = w.shape[1]
    idx = np.array([[mmac_index(H, r, k) for k in range(H)] for r in range(4 * H)])
    assert sorted(idx.ravel().tolist()) == list(range(4 * H * H))
    assert np.array_equal(packed[idx], w)


REFERENCE_C_FUNCTIONS = [  # miopen_adaptive_lstm_hip/csrc/bindings.cpp:6-78
    "adaptive_lstm_hidden_update_forward", "adaptive_lstm_hidden_update_partitioned_forward",
    "adaptive_lstm_h128_cached_update_forward", "adaptive_lstm_h128_cached_b4_update_forward",
    "adaptive_lstm_h128_cached_b8_update_forward", "adaptive_lstm_h128_gemm_scan_update_forward",
    "adaptive_lstm_h128_gemm_scan_update_forward_workspace", "adaptive_lstm_h128_seqmajor_accum_update_forward",
    "adaptive_lstm_input_gemm_forward_workspace", "adaptive_lstm_h256_gemm_scan_update_forward_workspace",
    "adaptive_lstm_h512_gemm_scan_update_forward_workspace", "adaptive_lstm_h256_gate_accum_update_forward_workspace",
    "adaptive_lstm_h512_gate_accum_update_forward_workspace",
    "adaptive_lstm_h128_persistent_mmac_update_forward_workspace",
    "adaptive_lstm_h128_mmac_packed_variant_forward_workspace",
    "adaptive_lstm_h256_mmac_packed_variant_forward_workspace",
    "adaptive_lstm_h512_mmac_packed_variant_forward_workspace", "adaptive_lstm_gemm_scan_update_forward_workspace",
]


def test_adaptive_extension_surface():
    plstm.install_aliases()
    import miopen_adaptive_lstm_hip
    import miopen_adaptive_lstm_hip._C as C

    for name in REFERENCE_C_FUNCTIONS:
        assert callable(getattr(C, name)), name
    for name in ("AdaptiveLSTMRegressor", "NativeModuleFallback", "convert_regressor_module"):
        assert hasattr(miopen_adaptive_lstm_hip, name), name
