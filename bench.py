#!/usr/bin/env python
"""Benchmark of the fused LSTM + Linear inference forward (one JSON line on rank 0).

Workload: the reference's LSTMRegressor — nn.LSTM(5, 128,
4, batch_first) + nn.Linear(128, 24) on the last step — batch 512 rows per GPU,
sequence 1000, f16 weights/activations with f32 accumulation, PyTorch-default
random weights (seed 0) and x ~ N(0, 1) (seed 1 + rank), uniform lengths.  A
step is one forward of the converted module (`convert_regressor_module(model)(x)`,
the reference's drop-in call) over one batch.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

For N > 1 it runs under torch.distributed.run, one process per GPU; each rank
forwards its own 512-row batch shard (weak scaling, weights replicated) and the
[512, 24] outputs are all-gathered (the only collective of the path, the final
output gather).  `--impl reference` times the reference path's CPU
implementation (the C oracle port of reference.py, f32, all host threads) on
rank 0 only.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

B_PER_GPU, T, I, H, L, O = 512, 1000, 5, 128, 4, 24
METRIC = "seq-timesteps/sec and wall s for 4L H128 LSTM+Linear b512 s1000 fp16, 1/2/4/8 B200"
UNIT = "seq-timesteps/s"
# Reference's headline: 3.08 s per 100 forwards of B=512, T=1000 on a Hygon K100_AI
# (persistent_lstm_hip/README.md:12) = 512 * 1000 * 100 / 3.08 seq-timesteps/s.
PUBLISHED = 512 * 1000 * 100 / 3.08
FALLBACK_PEAK_TFLOPS = 1590.0


def flops_per_forward(B: int, Tn: int, mode: str) -> float:
    per_ts = 2 * 4 * H * (I + H) + (L - 1) * 2 * 4 * H * (2 * H)
    lin = 2 * H * O * (B * Tn if mode == "seq" else B)
    return float(per_ts) * B * Tn + lin


def workload_config(n: int) -> dict:
    return {
        "workload": "cfg2: LSTMRegressor 4L LSTM(5->128)+Linear(128->24) forward -> [B,24], "
                    "b512/GPU s1000 f16 (f32 accumulate), uniform lengths",
        "model": "LSTM(5,128,4,batch_first)+Linear(128,24)",
        "global_batch": B_PER_GPU * n,
        "seq_len": T,
        "parallelism": f"dp{n} (batch shards, weights replicated, final output all-gather)",
        "l2": "flushed between timed steps (256 MiB device memset, untimed)",
    }


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.samples = []
        self.proc = None
        self.thread = None
        self.window = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-i",
                 str(self.index), "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.samples.append((time.time(), [v.strip() for v in line.split(",")]))

    def mark(self, t0, t1):
        self.window = (t0, t1)

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = self.samples
        inside = [r for t, r in rows if self.window and self.window[0] <= t <= self.window[1] + 0.1]
        use = inside or [r for _, r in rows[-5:]]
        sm = [float(r[1]) for r in use if len(r) >= 9 and r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in use if len(r) >= 9 and r[2].replace(".", "").isdigit()]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in use:
            if len(r) >= 9:
                for name, v in zip(names, r[5:9]):
                    if v.lower().startswith("active"):
                        reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples_in_timed_region": len(inside),
                "power_w_max": max((float(r[3]) for r in use if len(r) >= 9 and _isnum(r[3])), default=None)}


def _isnum(s: str) -> bool:
    try:
        float(s)
        return True
    except ValueError:
        return False


def measured_peak():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["bf16_tflops"]), "of measured (MEASURED_PEAKS.json bf16_tflops, burst)"
    except (OSError, KeyError, ValueError):
        return FALLBACK_PEAK_TFLOPS, "of fallback"


def profiled_traffic():
    """Per-launch DRAM bytes of the recurrent kernel from the committed ncu summary, if any."""
    path = os.path.join(ROOT, "profiles", "wavefront2_kernel_cfg2.md")
    try:
        for line in open(path):
            if line.startswith("traffic_bytes_per_launch:"):
                return int(line.split(":", 1)[1].strip())
    except (OSError, ValueError):
        pass
    return None


# ---------------------------------------------------------------------------------------
def cpu_oracle_sample(seconds: float = 10.0):
    """The reference path's CPU implementation (C port of reference.py, f32, all host
    threads) on a bounded sample of the workload: B=512 rows, the first Ts steps."""
    import numpy as np
    import torch
    import torch.nn as nn

    from oracle import oracle

    torch.manual_seed(0)
    lstm = nn.LSTM(I, H, L, batch_first=True)
    lin = nn.Linear(H, O)
    x = torch.randn(B_PER_GPU, T, I, generator=torch.Generator().manual_seed(1)).numpy()
    f = lambda t: t.detach().numpy().astype(np.float32)
    w_ih = [f(getattr(lstm, f"weight_ih_l{l}")) for l in range(L)]
    w_hh = [f(getattr(lstm, f"weight_hh_l{l}")) for l in range(L)]
    b_ih = [f(getattr(lstm, f"bias_ih_l{l}")) for l in range(L)]
    b_hh = [f(getattr(lstm, f"bias_hh_l{l}")) for l in range(L)]
    threads = os.cpu_count() or 1

    def run(ts):
        t0 = time.perf_counter()
        oracle.forward(x[:, :ts], w_ih, w_hh, b_ih, b_hh, f(lin.weight), f(lin.bias), out_mode="last",
                       precision="f32", threads=threads)
        return time.perf_counter() - t0

    dt = run(2)
    ts = int(max(2, min(T, seconds / max(dt / 2, 1e-6))))
    dt = run(ts)
    return {"value": B_PER_GPU * ts / dt, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"B=512 rows x first {ts} of 1000 steps, f32, oracle/plstm_oracle.c "
                      f"(C restatement of reference.py:11-72), {threads} OpenMP threads, {dt:.2f} s",
            "s_per_forward_extrapolated": dt * T / ts}


def run_reference(args, rank: int, world: int):
    if rank != 0:
        return
    import torch  # noqa: F401

    steps = []
    for k in range(args.warmup + args.steps):
        cb = cpu_oracle_sample(seconds=args.ref_step_seconds)
        if k >= args.warmup:
            steps.append(cb)
    vals = [c["value"] for c in steps]
    value = statistics.median(vals)
    cb = dict(steps[-1])
    cb["value"] = value
    ms = B_PER_GPU * T / value * 1e3
    line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded N(0,1) x, PyTorch-default init)",
            "config": workload_config(1), "impl": "reference", "cpu_baseline": cb,
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------------------
def run_ours(args, rank: int, world: int, local_rank: int):
    import ctypes

    import torch
    import torch.distributed as dist
    import torch.nn as nn

    import persistent_lstm_hip_b200 as plstm
    from persistent_lstm_hip_b200 import _lib

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    lib = _lib.load()

    class LSTMRegressor(nn.Module):
        def __init__(self):
            super().__init__()
            self.lstm = nn.LSTM(I, H, L, batch_first=True, dropout=0.2)
            self.linear = nn.Linear(H, O)

    torch.manual_seed(0)
    native = LSTMRegressor().eval().to(dev).half()
    model = plstm.convert_regressor_module(native)
    g = torch.Generator().manual_seed(1 + rank)
    x_host = torch.randn(B_PER_GPU, T, I, generator=g).half().pin_memory()
    x = x_host.to(dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    gathered = torch.empty(world * B_PER_GPU, O, dtype=torch.float16, device=dev) if world > 1 else None
    stream = torch.cuda.current_stream(dev)

    def step(xin):
        out = model(xin)
        if world > 1:
            dist.all_gather_into_tensor(gathered, out)
        return out

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local_rank])
        torch.cuda.synchronize(dev)

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    sampler = ClockSampler(local_rank if "CUDA_VISIBLE_DEVICES" not in os.environ else
                           int(os.environ["CUDA_VISIBLE_DEVICES"].split(",")[local_rank]))
    sampler.start()
    for _ in range(args.warmup):
        step(x)
    # ---- device-resident timing (value) ----
    lib.plstm_profile(1)
    ms_buf = ctypes.c_float(0)
    nl = ctypes.c_int32(0)
    lib.plstm_profile_read(ctypes.byref(ms_buf), ctypes.byref(nl))  # clear
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    barrier()
    launches0 = lib.plstm_launch_count()
    wall0 = time.time()
    for k in range(args.steps):
        flush.zero_()
        ev[k][0].record(stream)
        out = step(x)
        ev[k][1].record(stream)
    barrier()
    wall1 = time.time()
    sampler.mark(wall0, wall1)
    launches = lib.plstm_launch_count() - launches0
    _lib.check(lib.plstm_profile_read(ctypes.byref(ms_buf), ctypes.byref(nl)))
    lib.plstm_profile(0)
    step_ms = [a.elapsed_time(b) for a, b in ev]
    total_ms = max_over_ranks(sum(step_ms))
    ms_per_step = total_ms / args.steps
    kernel_ms = max_over_ranks(ms_buf.value / max(nl.value, 1))
    value = world * B_PER_GPU * T / (ms_per_step / 1e3)

    # ---- end to end through the public API with host buffers ----
    x_dev = torch.empty_like(x)
    out_host = torch.empty(B_PER_GPU, O, dtype=torch.float16).pin_memory()

    def e2e_step():
        x_dev.copy_(x_host, non_blocking=True)
        o = step(x_dev)
        out_host.copy_(o, non_blocking=True)

    for _ in range(max(1, args.warmup // 2)):
        e2e_step()
    ev2 = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    barrier()
    for k in range(args.steps):
        flush.zero_()
        ev2[k][0].record(stream)
        e2e_step()
        ev2[k][1].record(stream)
    barrier()
    e2e_ms = max_over_ranks(sum(a.elapsed_time(b) for a, b in ev2)) / args.steps
    clocks = sampler.stop()

    # ---- latency floor of one dependent wavefront step (single 16-row cluster) ----
    lat = None
    if rank == 0 and not args.no_latency:
        xs = x[:16].contiguous()
        for _ in range(3):
            model(xs)
        lib.plstm_profile(1)
        lib.plstm_profile_read(ctypes.byref(ms_buf), ctypes.byref(nl))
        for _ in range(10):
            model(xs)
        torch.cuda.synchronize(dev)
        lib.plstm_profile_read(ctypes.byref(ms_buf), ctypes.byref(nl))
        lib.plstm_profile(0)
        k16 = ms_buf.value / max(nl.value, 1)
        t_step_us = k16 * 1e3 / (T + L)
        bound_ms = t_step_us * (T + L) / 1e3
        lat = {"t_step_us": t_step_us, "steps": T + L,
               "method": "same kernel, B=16 (one 8-CTA cluster, one active 16-row slot), T=1000, "
                         "CUDA events, 10 runs",
               "bound_ms": bound_ms, "frac": bound_ms / kernel_ms}

    if rank != 0:
        return
    # Parity spot check of the timed output against the oracle (4 rows).
    cb = None
    if world == 1 and not args.no_cpu_baseline:
        cb = cpu_oracle_sample(seconds=args.cpu_seconds)
    peak, peak_note = measured_peak()
    flops = flops_per_forward(B_PER_GPU, T, "last")
    achieved = flops / (kernel_ms / 1e3) / 1e12
    roof = {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
            "traffic": profiled_traffic(), "kernel": "plstm::tc::wavefront2_kernel", "kernel_ms": kernel_ms,
            "peak_note": peak_note,
            "algorithmic_flops_per_launch": flops,
            "latency": lat}
    line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_per_step, "wall_s_per_100_forwards": ms_per_step / 10.0,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": value / PUBLISHED, "dtype": "f16",
            "data": "synthetic (seeded N(0,1) x, PyTorch-default init weights)", "config": workload_config(world),
            "roofline": roof, "cpu_baseline": cb,
            "e2e": {"value": world * B_PER_GPU * T / (e2e_ms / 1e3), "unit": UNIT,
                    "h2d_bytes_per_step": x_host.numel() * 2, "d2h_bytes_per_step": out_host.numel() * 2,
                    "ms_per_step": e2e_ms,
                    "call": "persistent_lstm_hip_b200.convert_regressor_module(model)(x) with pinned host x"},
            "gpu_launches": int(launches), "gpu_launches_per_step": launches / args.steps,
            "clocks": clocks, "backend": model.backend_name}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-latency", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--ref-step-seconds", type=float, default=1.0)
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        ap.error(f"--gpus {args.gpus} but WORLD_SIZE={world}; launch N>1 with torch.distributed.run")
    if args.impl == "reference":
        run_reference(args, rank, world)
        return
    if world > 1:
        import datetime

        import torch
        import torch.distributed as dist

        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                device_id=torch.device("cuda", local_rank))
    try:
        run_ours(args, rank, world, local_rank)
    finally:
        if world > 1:
            import torch.distributed as dist

            dist.destroy_process_group()


if __name__ == "__main__":
    main()
