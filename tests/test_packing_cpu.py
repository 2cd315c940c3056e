"""Host-side layout helpers against the reference's own packing outputs."""
from __future__ import annotations

import numpy as np
import torch

from conftest import load_golden
from persistent_lstm_hip_b200.packing import pack_recurrent_weight_kpairs, unpack_recurrent_weight_kpairs


def test_kpair_pack_matches_reference_odd_k():
    g = load_golden("ref_kpair_odd")
    got = pack_recurrent_weight_kpairs(torch.from_numpy(g["weight"]))
    np.testing.assert_array_equal(got.numpy(), g["packed"])


def test_kpair_pack_matches_reference_even_k():
    g = load_golden("ref_kpair_even")
    got = pack_recurrent_weight_kpairs(torch.from_numpy(g["weight"]))
    np.testing.assert_array_equal(got.numpy(), g["packed"])


def test_kpair_roundtrip():
    for name, k in (("ref_kpair_odd", 5), ("ref_kpair_even", 8)):
        g = load_golden(name)
        back = unpack_recurrent_weight_kpairs(torch.from_numpy(g["packed"]), k)
        np.testing.assert_array_equal(back.numpy(), g["weight"])
