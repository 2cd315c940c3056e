"""Microbenchmarks of the library's kernels (CUDA-event timed, one JSON line each).

    python -m persistent_lstm_hip_b200.microbench gemm [--m 512000 --k 5 --n 512]
        The input-projection GEMM (plstm_input_gemm) at the layer-0 shape of
        config 2 (x[B*T, I] . W_ih^T for B=512, T=1000, I=5, 4H=512): achieved HBM
        GB/s over its algorithmic bytes (read M*K + K*N, write M*N 16-bit values)
        and TFLOP/s over 2*M*N*K.
    python -m persistent_lstm_hip_b200.microbench step [--batch 16 --seq 1000]
        The recurrent wavefront kernel on one cluster: per-step latency floor.
    python -m persistent_lstm_hip_b200.microbench forward [--hidden 512 --layers 4 --batch 512
            --seq 1000 --input 5 --dtype bf16 --out last]
        One whole forward (lstm_linear_forward's packed call, PyTorch-default weights,
        N(0, 1) x) of any shape: configs 3 and 4, the generic shapes, the [B,T,O] mode.
    python -m persistent_lstm_hip_b200.microbench probe [--rows 16 --steps 20000]
        The dependent-step latency probe (plstm_diag_step_latency): one wavefront
        layer-step's dependency chain alone, cycles and microseconds per step and
        its phases; the latency floor of the roofline.
"""
from __future__ import annotations

import argparse
import ctypes
import json

import torch


def _time(fn, iters: int, warmup: int) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(iters)]
    for a, b in ev:
        a.record()
        fn()
        b.record()
    torch.cuda.synchronize()
    return sorted(a.elapsed_time(b) for a, b in ev)[iters // 2]


def gemm(args) -> dict:
    from .adaptive_ext import adaptive_lstm_input_gemm_forward_workspace

    dev = torch.device("cuda:0")
    g = torch.Generator().manual_seed(0)
    x = torch.randn(args.m, args.k, generator=g).to(dev, torch.float16)
    w = (torch.rand(args.k, args.n, generator=g) * 0.2 - 0.1).to(dev, torch.float16)
    gate = torch.empty(args.m, args.n, device=dev, dtype=torch.float16)
    ms = _time(lambda: adaptive_lstm_input_gemm_forward_workspace(x, w, gate), args.iters, 3)
    nbytes = 2 * (args.m * args.k + args.k * args.n + args.m * args.n)
    flops = 2.0 * args.m * args.n * args.k
    return {"kernel": "plstm::gemm::input_gemm_kernel", "m": args.m, "k": args.k, "n": args.n, "ms": ms,
            "algorithmic_bytes": nbytes, "gbs": nbytes / ms / 1e6, "tflops": flops / ms / 1e9}


def step(args) -> dict:
    from . import _lib, core

    dev = torch.device("cuda:0")
    torch.manual_seed(0)
    lstm = torch.nn.LSTM(5, 128, 4, batch_first=True)
    lin = torch.nn.Linear(128, 24)
    h = lambda t: t.detach().to(dev, torch.float16).contiguous()
    pw = core.PackedWeights([h(getattr(lstm, f"weight_ih_l{l}")) for l in range(4)],
                            [h(getattr(lstm, f"weight_hh_l{l}")) for l in range(4)],
                            [h(getattr(lstm, f"bias_ih_l{l}")) for l in range(4)],
                            [h(getattr(lstm, f"bias_hh_l{l}")) for l in range(4)], h(lin.weight), h(lin.bias),
                            out_mode="last")
    x = torch.randn(args.batch, args.seq, 5, device=dev).half()
    lib = _lib.load()
    for _ in range(3):
        pw.forward(x, need_state=False)
    lib.plstm_profile(1)
    ms, n = ctypes.c_float(0), ctypes.c_int32(0)
    lib.plstm_profile_read(ctypes.byref(ms), ctypes.byref(n))
    for _ in range(args.iters):
        pw.forward(x, need_state=False)
    torch.cuda.synchronize()
    lib.plstm_profile_read(ctypes.byref(ms), ctypes.byref(n))
    lib.plstm_profile(0)
    k_ms = ms.value / max(n.value, 1)
    return {"kernel": "plstm::tc::wavefront_kernel", "batch": args.batch, "seq": args.seq, "ms": k_ms,
            "us_per_step": k_ms * 1e3 / (args.seq + 4)}


def step_latency(rows: int = 16, steps: int = 20000, device: int = 0, variant: int = 0) -> dict:
    """The dependent-step latency probe (plstm_diag_step_latency): cycles and microseconds of one
    wavefront layer-step's dependency chain run alone, with its phases."""
    from . import _lib

    dev = torch.device("cuda", device)
    lib = _lib.load()
    out = torch.zeros(16, dtype=torch.int64, device=dev)
    stream = torch.cuda.current_stream(dev)
    for _ in range(2):  # warm-up (module load, clocks)
        _lib.check(lib.plstm_diag_step_latency(rows, 1000, variant, out.data_ptr(), 0, stream.cuda_stream))
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    _lib.check(lib.plstm_diag_step_latency(rows, steps, variant, out.data_ptr(), 0, stream.cuda_stream))
    b.record(stream)
    torch.cuda.synchronize(dev)
    o = [int(v) for v in out.cpu().tolist()]
    if o[0] != 0:
        raise _lib.PlstmError(_lib.ETIMEOUT, "step-latency probe: a bounded wait gave up")
    n = max(o[2], 1)
    phases = ["landed->commit issued", "commit->accumulator seen", "seen->loaded", "loaded->h written",
              "h written->copy issued", "copy issued->next h landed"]
    return {"rows": rows, "steps": steps, "variant": variant, "cycles_per_step": o[1] / n,
            "us_per_step": a.elapsed_time(b) * 1e3 / steps,
            "phase_cycles": {k: o[3 + i] / n for i, k in enumerate(phases)},
            "method": "plstm_diag_step_latency: 2-CTA cluster; per step the sibling's h lands, 8 tcgen05 MMAs "
                      "(2 x M128, K64, N=rows) + commit, tcgen05.ld, the kernel's gate math, h to shared memory, "
                      "one bulk DSMEM copy to the sibling; CUDA events over the launch / steps"}


def probe(args) -> dict:
    return step_latency(args.rows, args.steps, variant=args.variant)


def forward(args) -> dict:
    from . import core

    dev = torch.device("cuda:0")
    dt = {"f16": torch.float16, "bf16": torch.bfloat16, "f32": torch.float32}[args.dtype]
    torch.manual_seed(0)
    lstm = torch.nn.LSTM(args.input, args.hidden, args.layers, batch_first=True)
    lin = torch.nn.Linear(args.hidden, 24)
    h = lambda t: t.detach().to(dev, dt).contiguous()
    L = args.layers
    pw = core.PackedWeights([h(getattr(lstm, f"weight_ih_l{l}")) for l in range(L)],
                            [h(getattr(lstm, f"weight_hh_l{l}")) for l in range(L)],
                            [h(getattr(lstm, f"bias_ih_l{l}")) for l in range(L)],
                            [h(getattr(lstm, f"bias_hh_l{l}")) for l in range(L)], h(lin.weight), h(lin.bias),
                            out_mode=args.out)
    gen = torch.Generator().manual_seed(1)
    x = torch.randn(args.batch, args.seq, args.input, generator=gen).to(dev, dt)
    lengths = None
    steps = args.batch * args.seq
    if args.min_len is not None:  # lengths uniform in [min_len, seq], seeded (config 5 draws from [200, 1000])
        lengths = torch.randint(args.min_len, args.seq + 1, (args.batch,), generator=gen, dtype=torch.int32)
        steps = int(lengths.sum())
        lengths = lengths.to(dev)
    ms = _time(lambda: pw.forward(x, lengths=lengths, need_state=False), args.iters, 2)
    # The recurrent kernel alone (plstm_profile: CUDA events around its launches, mean).
    from . import _lib
    lib = _lib.load()
    lib.plstm_profile(1)
    k_ms, n = ctypes.c_float(0), ctypes.c_int32(0)
    lib.plstm_profile_read(ctypes.byref(k_ms), ctypes.byref(n))
    for _ in range(args.iters):
        pw.forward(x, lengths=lengths, need_state=False)
    torch.cuda.synchronize()
    lib.plstm_profile_read(ctypes.byref(k_ms), ctypes.byref(n))
    lib.plstm_profile(0)
    return {"backend": pw.backend, "hidden": args.hidden, "layers": L, "batch": args.batch, "seq": args.seq,
            "input": args.input, "dtype": args.dtype, "out": args.out, "min_len": args.min_len, "ms": ms,
            "kernel_ms": k_ms.value / max(n.value, 1), "seq_timesteps_per_s": steps / (ms / 1e3)}


def main() -> None:
    ap = argparse.ArgumentParser()
    sub = ap.add_subparsers(dest="cmd", required=True)
    g = sub.add_parser("gemm")
    g.add_argument("--m", type=int, default=512 * 1000)
    g.add_argument("--k", type=int, default=5)
    g.add_argument("--n", type=int, default=512)
    g.add_argument("--iters", type=int, default=20)
    s = sub.add_parser("step")
    s.add_argument("--batch", type=int, default=16)
    s.add_argument("--seq", type=int, default=1000)
    s.add_argument("--iters", type=int, default=10)
    f = sub.add_parser("forward")
    f.add_argument("--hidden", type=int, default=128)
    f.add_argument("--layers", type=int, default=4)
    f.add_argument("--batch", type=int, default=512)
    f.add_argument("--seq", type=int, default=1000)
    f.add_argument("--input", type=int, default=5)
    f.add_argument("--dtype", choices=["f16", "bf16", "f32"], default="f16")
    f.add_argument("--out", choices=["last", "seq", "hseq"], default="last")
    f.add_argument("--iters", type=int, default=5)
    f.add_argument("--min-len", type=int, default=None,
                   help="variable lengths uniform in [min_len, seq]; throughput counts the valid steps")
    pr = sub.add_parser("probe")
    pr.add_argument("--rows", type=int, choices=[16, 32], default=16)
    pr.add_argument("--steps", type=int, default=20000)
    pr.add_argument("--variant", type=int, default=0, help="bits of plstm_diag_step_latency's variants")
    args = ap.parse_args()
    print(json.dumps({"gemm": gemm, "step": step, "forward": forward, "probe": probe}[args.cmd](args)))


if __name__ == "__main__":
    main()
