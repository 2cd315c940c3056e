"""Generates the golden vectors in tests/golden/*.npz.

Run in a container that holds the reference checkout (read-only):

    python tests/golden/make_golden.py /path/to/persistent_lstm_hip_reference

The `ref_*` fixtures are outputs of the reference's own CPU implementation,
imported from its sources:
  * reference_lstm_forward        persistent_lstm_hip/persistent_lstm_hip/reference.py:11-63
  * reference_regressor_forward   persistent_lstm_hip/persistent_lstm_hip/reference.py:66-72
  * pack_lstm_module              persistent_lstm_hip/persistent_lstm_hip/packing.py:38-63
  * _pack_recurrent_weight_kpairs persistent_lstm_hip/persistent_lstm_hip/model.py:20-27
  * _pack_mmac_weight             miopen_adaptive_lstm_hip/miopen_adaptive_lstm_hip/model.py:259-286
The `torch_varlen` fixture (variable lengths, which the reference has no path
for) comes from torch.nn.LSTM + pack_padded_sequence, the semantics the
north star defines the masked path by.

Weights are PyTorch's default nn.LSTM / nn.Linear initialisation under a fixed
seed; inputs are seeded N(0, 1).  Nothing here is needed at test time: the
tests only read the .npz files.
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def _import_reference(root: str):
    sys.dont_write_bytecode = True  # never write into the reference checkout
    sys.path.insert(0, os.path.join(root, "persistent_lstm_hip"))
    from persistent_lstm_hip import model as ref_model  # noqa: E402
    from persistent_lstm_hip import packing as ref_packing  # noqa: E402
    from persistent_lstm_hip import reference as ref_reference  # noqa: E402
    return ref_model, ref_packing, ref_reference


def _module(I, H, L, O, dtype, seed):
    import torch
    import torch.nn as nn

    torch.manual_seed(seed)

    class Regressor(nn.Module):
        def __init__(self):
            super().__init__()
            self.lstm = nn.LSTM(I, H, L, batch_first=True)
            self.linear = nn.Linear(H, O)

    return Regressor().to(dtype).eval()


def _weights(m, L):
    d = {}
    for l in range(L):
        for n in ("weight_ih", "weight_hh", "bias_ih", "bias_hh"):
            d[f"{n}_l{l}"] = getattr(m.lstm, f"{n}_l{l}").detach().numpy().copy()
    d["linear_weight"] = m.linear.weight.detach().numpy().copy()
    d["linear_bias"] = m.linear.bias.detach().numpy().copy()
    return d


def make_reference_case(refs, name, I, H, L, O, B, T, dtype, seed, with_state):
    import torch

    ref_model, ref_packing, ref_reference = refs
    m = _module(I, H, L, O, dtype, seed)
    g = torch.Generator().manual_seed(seed + 1)
    x = torch.randn(B, T, I, generator=g, dtype=torch.float64).to(dtype)
    state = None
    arrays = {}
    if with_state:
        h0 = (0.5 * torch.randn(L, B, H, generator=g, dtype=torch.float64)).to(dtype)
        c0 = (0.5 * torch.randn(L, B, H, generator=g, dtype=torch.float64)).to(dtype)
        state = (h0, c0)
        arrays["h0"] = h0.numpy()
        arrays["c0"] = c0.numpy()
    with torch.no_grad():
        packed = ref_packing.pack_regressor_module(m)
        out, (h_n, c_n) = ref_reference.reference_lstm_forward(x, packed.lstm, state=state)
        reg = ref_reference.reference_regressor_forward(x, packed) if not with_state else None
    arrays.update(_weights(m, L))
    arrays.update(x=x.numpy(), out_h=out.numpy(), h_n=h_n.numpy(), c_n=c_n.numpy(),
                  dims=np.array([B, T, I, H, L, O], dtype=np.int64))
    if reg is not None:
        arrays["regressor_out"] = reg.numpy()
    np.savez_compressed(os.path.join(HERE, name + ".npz"), **arrays)


def make_kpair_case(refs, name, H, K, seed):
    import torch

    ref_model = refs[0]
    g = torch.Generator().manual_seed(seed)
    w = torch.randn(4 * H, K, generator=g, dtype=torch.float32).half()
    packed = ref_model._pack_recurrent_weight_kpairs(w)
    np.savez_compressed(os.path.join(HERE, name + ".npz"), weight=w.numpy(),
                        packed=packed.numpy())


def make_mmac_case(root, name, H, seed):
    import torch

    sys.dont_write_bytecode = True  # never write into the reference checkout
    sys.path.insert(0, os.path.join(root, "miopen_adaptive_lstm_hip"))
    from miopen_adaptive_lstm_hip import model as ada_model  # noqa: E402

    g = torch.Generator().manual_seed(seed)
    w = torch.randn(4 * H, H, generator=g, dtype=torch.float32).half()
    packed = ada_model._pack_mmac_weight(w, H)
    np.savez_compressed(os.path.join(HERE, name + ".npz"), weight=w.numpy(), packed=packed.numpy())


def make_varlen_case(name, I, H, L, O, B, T, seed):
    import torch
    from torch.nn.utils.rnn import pack_padded_sequence, pad_packed_sequence

    m = _module(I, H, L, O, torch.float64, seed)
    g = torch.Generator().manual_seed(seed + 1)
    x = torch.randn(B, T, I, generator=g, dtype=torch.float64)
    lengths = torch.randint(1, T + 1, (B,), generator=g)
    lengths[0] = T
    with torch.no_grad():
        packed = pack_padded_sequence(x, lengths, batch_first=True, enforce_sorted=False)
        out_p, (h_n, c_n) = m.lstm(packed)
        out_h, _ = pad_packed_sequence(out_p, batch_first=True, padding_value=0.0, total_length=T)
        y = m.linear(out_h)
        mask = (torch.arange(T)[None, :] < lengths[:, None]).unsqueeze(-1)
        y = torch.where(mask, y, torch.zeros_like(y))
    arrays = _weights(m, L)
    arrays.update(x=x.numpy(), lengths=lengths.numpy().astype(np.int32), out_h=out_h.numpy(),
                  out_seq=y.numpy(), h_n=h_n.numpy(), c_n=c_n.numpy(),
                  dims=np.array([B, T, I, H, L, O], dtype=np.int64))
    np.savez_compressed(os.path.join(HERE, name + ".npz"), **arrays)


def main(root: str, only: str = "") -> None:
    import torch

    if only == "mmac":
        make_mmac_case(root, "ref_mmac_h32", H=32, seed=17)
        return
    refs = _import_reference(root)
    make_reference_case(refs, "ref_small_f64", I=5, H=16, L=2, O=4, B=3, T=7,
                        dtype=torch.float64, seed=11, with_state=False)
    make_reference_case(refs, "ref_state_f64", I=3, H=8, L=3, O=2, B=2, T=5,
                        dtype=torch.float64, seed=12, with_state=True)
    make_reference_case(refs, "ref_h128_f32", I=5, H=128, L=4, O=24, B=4, T=12,
                        dtype=torch.float32, seed=13, with_state=False)
    make_kpair_case(refs, "ref_kpair_odd", H=8, K=5, seed=14)
    make_kpair_case(refs, "ref_kpair_even", H=8, K=8, seed=15)
    make_varlen_case("torch_varlen_f64", I=5, H=16, L=2, O=4, B=5, T=9, seed=16)
    make_mmac_case(root, "ref_mmac_h32", H=32, seed=17)


if __name__ == "__main__":
    if len(sys.argv) not in (2, 3):
        sys.exit("usage: make_golden.py <reference checkout root> [mmac]")
    main(sys.argv[1], sys.argv[2] if len(sys.argv) == 3 else "")
