"""Pins the CPU oracle to the reference's own outputs (tests/golden/*.npz).

The ref_* fixtures were produced by the reference's reference_lstm_forward /
reference_regressor_forward (persistent_lstm_hip/persistent_lstm_hip/reference.py:11-72);
torch_varlen_f64 by torch.nn.LSTM over pack_padded_sequence.
"""
from __future__ import annotations

import numpy as np
import pytest

from conftest import golden_weights, load_golden
from oracle import oracle


@pytest.mark.parametrize("name", ["ref_small_f64", "ref_state_f64", "ref_h128_f32"])
@pytest.mark.parametrize("impl", ["c_f64", "numpy"])
def test_oracle_matches_reference_sequence(name, impl):
    g = load_golden(name)
    B, T, I, H, L, O = (int(v) for v in g["dims"])
    w_ih, w_hh, b_ih, b_hh, w_lin, b_lin = golden_weights(g, L)
    kw = dict(h0=g.get("h0"), c0=g.get("c0"), out_mode="hseq")
    if impl == "c_f64":
        out, h_n, c_n = oracle.forward(g["x"], w_ih, w_hh, b_ih, b_hh, None, None, **kw)
    else:
        out, h_n, c_n = oracle.forward_numpy(g["x"], w_ih, w_hh, b_ih, b_hh, None, None, **kw)
    tol = 1e-12 if g["x"].dtype == np.float64 else 2e-6
    np.testing.assert_allclose(out, g["out_h"], atol=tol, rtol=0)
    np.testing.assert_allclose(h_n, g["h_n"], atol=tol, rtol=0)
    np.testing.assert_allclose(c_n, g["c_n"], atol=tol, rtol=0)


@pytest.mark.parametrize("name", ["ref_small_f64", "ref_h128_f32"])
def test_oracle_matches_reference_regressor(name):
    g = load_golden(name)
    B, T, I, H, L, O = (int(v) for v in g["dims"])
    w_ih, w_hh, b_ih, b_hh, w_lin, b_lin = golden_weights(g, L)
    out, _, _ = oracle.forward(g["x"], w_ih, w_hh, b_ih, b_hh, w_lin, b_lin, out_mode="last")
    tol = 1e-12 if g["x"].dtype == np.float64 else 2e-6
    np.testing.assert_allclose(out, g["regressor_out"], atol=tol, rtol=0)
    seq, _, _ = oracle.forward(g["x"], w_ih, w_hh, b_ih, b_hh, w_lin, b_lin, out_mode="seq")
    np.testing.assert_allclose(seq[:, -1, :], g["regressor_out"], atol=tol, rtol=0)


def test_oracle_f32_close_to_reference():
    g = load_golden("ref_h128_f32")
    B, T, I, H, L, O = (int(v) for v in g["dims"])
    w_ih, w_hh, b_ih, b_hh, w_lin, b_lin = golden_weights(g, L)
    out, _, _ = oracle.forward(g["x"], w_ih, w_hh, b_ih, b_hh, w_lin, b_lin, out_mode="last",
                               precision="f32")
    np.testing.assert_allclose(out, g["regressor_out"], atol=1e-5, rtol=0)


@pytest.mark.parametrize("impl", ["c_f64", "numpy"])
def test_oracle_matches_torch_varlen(impl):
    g = load_golden("torch_varlen_f64")
    B, T, I, H, L, O = (int(v) for v in g["dims"])
    w_ih, w_hh, b_ih, b_hh, w_lin, b_lin = golden_weights(g, L)
    fn = oracle.forward if impl == "c_f64" else oracle.forward_numpy
    seq, h_n, c_n = fn(g["x"], w_ih, w_hh, b_ih, b_hh, w_lin, b_lin, lengths=g["lengths"], out_mode="seq")
    np.testing.assert_allclose(seq, g["out_seq"], atol=1e-12, rtol=0)
    np.testing.assert_allclose(h_n, g["h_n"], atol=1e-12, rtol=0)
    np.testing.assert_allclose(c_n, g["c_n"], atol=1e-12, rtol=0)
    hs, _, _ = fn(g["x"], w_ih, w_hh, b_ih, b_hh, None, None, lengths=g["lengths"], out_mode="hseq")
    np.testing.assert_allclose(hs, g["out_h"], atol=1e-12, rtol=0)
    last, _, _ = fn(g["x"], w_ih, w_hh, b_ih, b_hh, w_lin, b_lin, lengths=g["lengths"], out_mode="last")
    idx = g["lengths"] - 1
    np.testing.assert_allclose(last, g["out_seq"][np.arange(B), idx], atol=1e-12, rtol=0)


def test_oracle_zero_length_rows_keep_initial_state():
    rng = np.random.default_rng(0)
    B, T, I, H, L, O = 3, 4, 2, 4, 2, 3
    w_ih = [rng.standard_normal((4 * H, I if l == 0 else H)) * 0.3 for l in range(L)]
    w_hh = [rng.standard_normal((4 * H, H)) * 0.3 for _ in range(L)]
    b = [rng.standard_normal(4 * H) * 0.1 for _ in range(L)]
    h0 = rng.standard_normal((L, B, H))
    c0 = rng.standard_normal((L, B, H))
    x = rng.standard_normal((B, T, I))
    lens = np.array([0, 2, 4], dtype=np.int32)
    out, h_n, c_n = oracle.forward(x, w_ih, w_hh, b, None, rng.standard_normal((O, H)), np.zeros(O),
                                   lengths=lens, h0=h0, c0=c0, out_mode="seq")
    np.testing.assert_array_equal(out[0], 0.0)
    np.testing.assert_array_equal(h_n[:, 0], h0[:, 0])
    np.testing.assert_array_equal(c_n[:, 0], c0[:, 0])
    np.testing.assert_array_equal(out[1, 2:], 0.0)
    ref = oracle.forward_numpy(x, w_ih, w_hh, b, None, rng.standard_normal((O, H)), np.zeros(O),
                               lengths=lens, h0=h0, c0=c0, out_mode="hseq")
    got = oracle.forward(x, w_ih, w_hh, b, None, None, None, lengths=lens, h0=h0, c0=c0, out_mode="hseq")
    for a, r in zip(got, ref):
        np.testing.assert_allclose(a, r, atol=1e-12)


def test_unique_rows_restates_the_uniform_check():
    """All rows equal (the reference's torch.equal(x, x[:1].expand_as(x)),
    persistent_lstm_hip/model.py:515-518) <=> one distinct row; duplicates are
    numbered by first occurrence; padding past a length and hx rows count as
    the row's identity the way the forward reads them."""
    rng = np.random.default_rng(5)
    base = rng.standard_normal((1, 6, 3)).astype(np.float16)
    x = np.repeat(base, 4, axis=0)
    assert oracle.unique_rows(x)[2] == 1
    x[2, 5, 1] += np.float16(1.0)
    row_map, first, n = oracle.unique_rows(x)
    assert n == 2 and list(row_map) == [0, 0, 1, 0] and list(first) == [0, 2]
    # Row 2 differs only past its length 5: it joins row 0 (same length).
    row_map, _, n = oracle.unique_rows(x, lengths=[5, 6, 5, 6])
    assert list(row_map) == [0, 1, 0, 1] and n == 2
    h0 = np.zeros((2, 4, 8), dtype=np.float16)
    c0 = np.zeros_like(h0)
    c0[1, 3, 7] = 1.0
    row_map, _, n = oracle.unique_rows(x, lengths=[5, 6, 5, 6], h0=h0, c0=c0)
    assert list(row_map) == [0, 1, 0, 2] and n == 3


# ---- against the reference's own C++ CPU path (oracle/_ref, built from
# persistent_lstm_hip/csrc/persistent_lstm_reference.cpp by oracle/build_ref.py) ----
def _ref_or_skip():
    from oracle import ref

    if not ref.available():
        pytest.skip("oracle/_ref/libplstm_ref.so is not built (needs the reference checkout at build time)")
    return ref


def _cfg2_like_weights(seed, I=5, H=128, O=24):
    rng = np.random.default_rng(seed)
    k = 1.0 / np.sqrt(H)
    u = lambda *s: rng.uniform(-k, k, size=s)
    w_ih = [u(4 * H, I if l == 0 else H) for l in range(4)]
    w_hh = [u(4 * H, H) for _ in range(4)]
    b_ih = [u(4 * H) for _ in range(4)]
    b_hh = [u(4 * H) for _ in range(4)]
    return w_ih, w_hh, b_ih, b_hh, u(O, H), u(O)


@pytest.mark.parametrize("B, T, I, H", [(6, 40, 5, 128), (3, 17, 7, 32)])
def test_oracle_matches_reference_cpp_path(B, T, I, H):
    """The C restatement equals persistent_lstm4_forward_reference (f64) on the same inputs."""
    ref = _ref_or_skip()
    w = _cfg2_like_weights(B * 131 + T, I=I, H=H)
    x = np.random.default_rng(7).standard_normal((B, T, I))
    got, _, _ = oracle.forward(x, *w, out_mode="last")
    want = ref.forward(x, *w, precision="f64", threads=2)
    np.testing.assert_allclose(got, want, atol=1e-12, rtol=0)


def test_oracle_matches_reference_cpp_path_cfg2_rows():
    """Config-2 shape (T = 1000 dependent steps) on 4 rows: f64 to 1e-12, and the f32
    restatement (the timed CPU port) within 1e-4 of the reference's f32 run."""
    ref = _ref_or_skip()
    w = _cfg2_like_weights(0)
    x = np.random.default_rng(1).standard_normal((4, 1000, 5))
    got, _, _ = oracle.forward(x, *w, out_mode="last")
    np.testing.assert_allclose(got, ref.forward(x, *w, precision="f64", threads=2), atol=1e-12, rtol=0)
    got32, _, _ = oracle.forward(x, *w, out_mode="last", precision="f32")
    np.testing.assert_allclose(got32, ref.forward(x, *w, precision="f32", threads=2), atol=1e-4, rtol=0)
