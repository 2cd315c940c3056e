#!/usr/bin/env python
"""Benchmark of the fused LSTM + Linear inference forward (one JSON line on rank 0).

Headline workload: the reference's LSTMRegressor — nn.LSTM(5, 128, 4, batch_first) +
nn.Linear(128, 24) on the last step — 512 rows per GPU, sequence 1000, f16 weights and
activations with f32 accumulation, PyTorch-default random weights (seed 0), x ~ N(0, 1)
(seed 1 + rank), uniform lengths.  A step is one forward of the converted module
(`convert_regressor_module(model)(x)`, the reference's drop-in call) over one batch.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

For N > 1 it runs under torch.distributed.run, one process per GPU; each rank forwards
its own 512-row shard (weak scaling, weights replicated) and the [512, 24] outputs are
all-gathered (the path's only collective, the final output gather).

The same line also carries, measured in the same run:
  * "strong_scaling": 4096 rows with lengths uniform in [200, 1000] (seed 2), [B, T, O]
    output zero past each length, dealt over the N ranks by shard.plan_shards (rows sorted
    by length and dealt round robin); each rank forwards its shard, the outputs are
    all-gathered.  value = valid seq-timesteps (the sum of the lengths) / max-over-ranks
    device time; at N = 1 one GPU runs all 4096 rows.
  * "configs" (N = 1): the 4-layer H = 256 (f16) and H = 512 (bf16) models at B = 512,
    T = 1000, [B, O] output.
  * "roofline": the recurrent kernel's FLOP rate against the measured dense bf16 peak and its
    time against the latency floor, (T + L - 1) x the dependent-step time of the probe
    kernel plstm_diag_step_latency (and T x L x that time, the layer-serial form).
  * "parity": rows of the timed output against the f64 oracle (the run fails outside the
    16-bit tolerance).
  * "cpu_baseline" (N = 1): torch.nn.LSTM + nn.Linear in f32 (the reference's CPU model,
    LSTM.py:9-27) full forwards on all host cores, 1 warm-up + median of 3, with the
    reference's own C++ CPU path (oracle/_ref) and the C restatement beside it.

`--impl reference` times that CPU model (full forwards of the headline workload, f32, all
host threads) on rank 0 only; the other ranks exit without work.
"""
from __future__ import annotations

import argparse
import json
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
STRONG_B, STRONG_MIN_LEN = 4096, 200
TOL16_MAX, TOL16_MEAN = 2e-2, 5e-3


def flops_per_forward(B: int, Tn: int, mode: str, hid: int = H, layers: int = L) -> float:
    per_ts = 2 * 4 * hid * (I + hid) + (layers - 1) * 2 * 4 * hid * (2 * hid)
    lin = 2 * hid * O * (B * Tn if mode == "seq" else B)
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
        sm = [float(r[1]) for r in use if len(r) >= 9 and _isnum(r[1])]
        mx = [float(r[2]) for r in use if len(r) >= 9 and _isnum(r[2])]
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


def cpu_model_name() -> str:
    try:
        for line in open("/proc/cpuinfo"):
            if line.lower().startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


# ---------------------------------------------------------------------------------------
# CPU baselines (the reference's CPU paths); test infrastructure under oracle/ is used only here.
def _cfg2_cpu_model():
    import torch
    import torch.nn as nn

    torch.manual_seed(0)
    lstm = nn.LSTM(I, H, L, batch_first=True).eval()
    lin = nn.Linear(H, O).eval()
    x = torch.randn(B_PER_GPU, T, I, generator=torch.Generator().manual_seed(1))
    return lstm, lin, x


def torch_cpu_forwards(n_timed: int, n_warm: int):
    """Full f32 forwards of the headline workload through torch.nn.LSTM + nn.Linear on all host
    cores (the reference's CPU model, LSTM.py:9-27); returns per-forward seconds."""
    import torch

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    lstm, lin, x = _cfg2_cpu_model()
    times = []
    with torch.inference_mode():
        for k in range(n_warm + n_timed):
            t0 = time.perf_counter()
            y, _ = lstm(x)
            lin(y[:, -1])
            dt = time.perf_counter() - t0
            if k >= n_warm:
                times.append(dt)
    return times, threads


def reference_cpp_forward():
    """One full f32 forward through the reference's own C++ CPU path (oracle/_ref), or None."""
    from oracle import ref

    if not ref.available():
        return None
    lstm, lin, x = _cfg2_cpu_model()
    f = lambda t: t.detach().numpy()
    w = [[f(getattr(lstm, f"{n}_l{l}")) for l in range(L)] for n in ("weight_ih", "weight_hh", "bias_ih", "bias_hh")]
    threads = os.cpu_count() or 1
    t0 = time.perf_counter()
    ref.forward(x.numpy(), *w, f(lin.weight), f(lin.bias), precision="f32", threads=threads)
    dt = time.perf_counter() - t0
    return {"value": B_PER_GPU * T / dt, "unit": UNIT, "cores": threads, "kind": "reference",
            "s_per_forward": dt,
            "sample": "one full B=512 T=1000 forward, f32, persistent_lstm4_forward_reference "
                      "(persistent_lstm_hip/csrc/persistent_lstm_reference.cpp:42-64, built as oracle/_ref)"}


def port_sample(seconds: float):
    """The C restatement of reference.py (oracle/plstm_oracle.c), f32, all host threads, on the
    first Ts steps of the headline batch (a bounded sample: every step costs the same)."""
    import numpy as np

    from oracle import oracle

    lstm, lin, x = _cfg2_cpu_model()
    xs = x.numpy()
    f = lambda t: t.detach().numpy().astype(np.float32)
    w = [[f(getattr(lstm, f"{n}_l{l}")) for l in range(L)] for n in ("weight_ih", "weight_hh", "bias_ih", "bias_hh")]
    threads = os.cpu_count() or 1

    def run(ts):
        t0 = time.perf_counter()
        oracle.forward(xs[:, :ts], *w, f(lin.weight), f(lin.bias), out_mode="last", precision="f32", threads=threads)
        return time.perf_counter() - t0

    dt = run(2)
    ts = int(max(2, min(T, seconds / max(dt / 2, 1e-6))))
    dt = run(ts)
    return {"value": B_PER_GPU * ts / dt, "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"B=512 rows x first {ts} of 1000 steps, f32, oracle/plstm_oracle.c "
                      f"(C restatement of reference.py:11-72), {threads} OpenMP threads, {dt:.2f} s"}


def cpu_baseline(port_seconds: float) -> dict:
    times, threads = torch_cpu_forwards(3, 1)
    med = statistics.median(times)
    cb = {"value": B_PER_GPU * T / med, "unit": UNIT, "cores": threads, "kind": "reference",
          "cpu_model": cpu_model_name(), "s_per_forward": med,
          "sample": f"torch.nn.LSTM(5,128,4)+nn.Linear(128,24) f32 (the reference's CPU model, LSTM.py:9-27), "
                    f"full B=512 T=1000 forwards on {threads} threads: 1 warm-up, median of 3 "
                    f"({', '.join(f'{t:.2f}' for t in times)} s)",
          "also": []}
    try:
        r = reference_cpp_forward()
        if r is not None:
            cb["also"].append(r)
    except Exception as exc:  # the baseline is reported, not required
        cb["also"].append({"kind": "reference", "error": str(exc)[:200]})
    cb["also"].append(port_sample(port_seconds))
    return cb


def run_reference(args, rank: int, world: int):
    if rank != 0:
        return
    times, threads = torch_cpu_forwards(args.steps, args.warmup)
    total = sum(times)
    value = B_PER_GPU * T * len(times) / total
    cb = {"value": value, "unit": UNIT, "cores": threads, "kind": "reference", "cpu_model": cpu_model_name(),
          "sample": f"torch.nn.LSTM(5,128,4)+nn.Linear(128,24) f32 (the reference's CPU model, LSTM.py:9-27), "
                    f"{len(times)} full B=512 T=1000 forwards after {args.warmup} warm-ups on {threads} threads, "
                    f"median {statistics.median(times):.3f} s"}
    line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": total / len(times) * 1e3, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded N(0,1) x, PyTorch-default init)", "config": workload_config(1),
            "impl": "reference", "cpu_baseline": cb,
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------------------
def spot_check(x, native, out, rows, mode="last", lengths=None) -> dict:
    """Rows of a timed output against the f64 oracle run on the same f16-rounded values."""
    import numpy as np
    import torch

    from oracle import oracle

    f = lambda t: t.detach().to("cpu", dtype=torch.float64).numpy()
    lstm, lin = native.lstm, native.linear
    nl = lstm.num_layers
    w = [[f(getattr(lstm, f"{n}_l{l}")) for l in range(nl)] for n in ("weight_ih", "weight_hh", "bias_ih", "bias_hh")]
    lens = None if lengths is None else lengths[rows].cpu().numpy().astype(np.int32)
    r_out, _, _ = oracle.forward(f(x[rows]), *w, f(lin.weight), f(lin.bias), lengths=lens, out_mode=mode)
    d = np.abs(f(out[rows]) - r_out)
    res = {"rows": [int(r) for r in rows], "max_abs": float(d.max()), "mean_abs": float(d.mean()),
           "tol_max": TOL16_MAX, "tol_mean": TOL16_MEAN}
    res["ok"] = res["max_abs"] <= TOL16_MAX and res["mean_abs"] <= TOL16_MEAN
    return res


def run_ours(args, rank: int, world: int, local_rank: int):
    import ctypes

    import torch
    import torch.distributed as dist
    import torch.nn as nn

    import persistent_lstm_hip_b200 as plstm
    from persistent_lstm_hip_b200 import _lib, microbench, shard

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    lib = _lib.load()

    class LSTMRegressor(nn.Module):
        def __init__(self, hid=H, layers=L):
            super().__init__()
            self.lstm = nn.LSTM(I, hid, layers, batch_first=True, dropout=0.2)
            self.linear = nn.Linear(hid, O)

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

    def timed(fn, steps):
        """Device time (ms) of each of `steps` calls on the current stream, L2 flushed before each."""
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        barrier()
        for k in range(steps):
            flush.zero_()
            ev[k][0].record(stream)
            fn()
            ev[k][1].record(stream)
        barrier()
        return [a.elapsed_time(b) for a, b in ev]

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
    out = None
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
    timed_out = out.clone()

    # ---- end to end through the public API with host buffers ----
    x_dev = torch.empty_like(x)
    out_host = torch.empty(B_PER_GPU, O, dtype=torch.float16).pin_memory()

    def e2e_step():
        x_dev.copy_(x_host, non_blocking=True)
        o = step(x_dev)
        out_host.copy_(o, non_blocking=True)

    for _ in range(max(1, args.warmup // 2)):
        e2e_step()
    e2e_ms = max_over_ranks(sum(timed(e2e_step, args.steps))) / args.steps
    clocks = sampler.stop()

    # ---- strong scaling: 4096 variable-length rows dealt over the ranks ----
    strong = None
    if not args.no_strong:
        lens_all = torch.randint(STRONG_MIN_LEN, T + 1, (STRONG_B,), generator=torch.Generator().manual_seed(2),
                                 dtype=torch.int32)
        x_all = torch.randn(STRONG_B, T, I, generator=torch.Generator().manual_seed(3)).half()
        plan = shard.plan_shards(STRONG_B, world, lens_all.tolist())
        idx = plan[rank]
        xs = x_all[idx].to(dev)
        ls = lens_all[idx].to(dev)
        rows_loc = int(idx.numel())
        seq_out = torch.empty(world * rows_loc, T, O, dtype=torch.float16, device=dev) if world > 1 else None
        res = {}

        def strong_step():
            o, _ = model.forward_sequence(xs, lengths=ls)
            res["out"] = o
            if world > 1:
                dist.all_gather_into_tensor(seq_out, o)

        def strong_compute():
            o, _ = model.forward_sequence(xs, lengths=ls)
            res["out"] = o

        for _ in range(args.warmup):
            strong_step()
        st_ms = max_over_ranks(statistics.median(timed(strong_step, args.steps)))
        comp_ms = max_over_ranks(statistics.median(timed(strong_compute, args.steps)))
        valid = int(lens_all.sum())
        strong = {"workload": "cfg5: 4096 rows, lengths uniform in [200, 1000] (seed 2), x seed 3, [B,T,O] f16 "
                              "zero past each length; rows length-sorted and dealt round robin over the ranks "
                              "(shard.plan_shards), each rank's shard forwarded, outputs all-gathered",
                  "global_batch": STRONG_B, "rows_per_gpu": rows_loc, "valid_timesteps": valid,
                  "ms": st_ms, "compute_ms": comp_ms,
                  "value": valid / (st_ms / 1e3), "unit": "valid seq-timesteps/s",
                  "padded_value": STRONG_B * T / (st_ms / 1e3),
                  "max_len_per_gpu": int(lens_all[idx].max()), "scaling": "strong",
                  "timing": "median over --steps of device time (CUDA events) of forward + all-gather, "
                            "max over ranks; compute_ms without the gather"}
        if rank == 0:
            o = res["out"]
            loc_rows = [0, rows_loc - 1]  # this rank's longest and shortest rows
            strong["parity"] = spot_check(xs, native, o, loc_rows, mode="seq", lengths=ls)
        del x_all

    # ---- configs 3 and 4 on one GPU ----
    configs = None
    if world == 1 and not args.no_configs:
        configs = {}
        peak, _ = measured_peak()
        for name, hid, dt in (("cfg3", 256, torch.float16), ("cfg4", 512, torch.bfloat16)):
            torch.manual_seed(0)
            nat = LSTMRegressor(hid).eval().to(dev).to(dt)
            mdl = plstm.convert_regressor_module(nat)
            xc = torch.randn(B_PER_GPU, T, I, generator=torch.Generator().manual_seed(1)).to(dev, dt)
            for _ in range(2):
                mdl(xc)
            ms = statistics.median(timed(lambda: mdl(xc), 5))
            fl = flops_per_forward(B_PER_GPU, T, "last", hid=hid)
            configs[name] = {"model": f"LSTM(5,{hid},4)+Linear({hid},24), B=512, T=1000, [B,O]",
                             "dtype": "bf16" if dt == torch.bfloat16 else "f16", "ms": ms,
                             "wall_s_per_100_forwards": ms / 10.0, "value": B_PER_GPU * T / (ms / 1e3),
                             "unit": UNIT, "tflops": fl / (ms / 1e3) / 1e12,
                             "frac_dense_peak": fl / (ms / 1e3) / 1e12 / peak, "backend": mdl.backend_name}
            del nat, mdl, xc
            torch.cuda.empty_cache()

    # ---- latency floor: the dependent-step probe ----
    lat = None
    if rank == 0 and not args.no_latency:
        probes = {r: microbench.step_latency(rows=r, steps=20000, device=local_rank) for r in (16, 32)}
        # The config-2 kernel runs 16-row slots (three per 48-row tile).  The probe's step in SM cycles,
        # at the SM clock sampled during the timed region (a lone 2-CTA launch may run at another clock).
        sm_mhz = clocks.get("sm_mhz") or 1965.0
        t_step = probes[16]["cycles_per_step"] / sm_mhz
        wave_ms = t_step * (T + L - 1) / 1e3
        serial_ms = t_step * T * L / 1e3
        lat = {"t_step_us": t_step, "probe": probes,
               "floor_wavefront_ms": wave_ms, "frac_wavefront": wave_ms / kernel_ms,
               "floor_layer_serial_ms": serial_ms, "frac_layer_serial": serial_ms / kernel_ms,
               "sm_mhz": sm_mhz,
               "method": "(T + L - 1) x t_step, t_step = the 16-row probe's cycles per step (the kernel's slot "
                         "height) at the SM clock sampled during the timed region (a wavefront of T + L - 1 "
                         "dependent steps); T x L x t_step is the north star's layer-serial form"}

    if rank != 0:
        return
    parity = spot_check(x, native, timed_out, [0, 171, 342, 511])
    cb = None
    if world == 1 and not args.no_cpu_baseline:
        cb = cpu_baseline(args.cpu_seconds)
    peak, peak_note = measured_peak()
    flops = flops_per_forward(B_PER_GPU, T, "last")
    achieved = flops / (kernel_ms / 1e3) / 1e12
    flop_ms = flops / (peak * 1e12) * 1e3
    if lat is not None and lat["floor_wavefront_ms"] > flop_ms:
        roof_ms, bound = lat["floor_wavefront_ms"], "latency"
    else:
        roof_ms, bound = flop_ms, "tensor"
    roof = {"bound": bound, "achieved": achieved, "peak": flops / (roof_ms / 1e3) / 1e12, "unit": "TFLOP/s",
            "frac": roof_ms / kernel_ms, "traffic": profiled_traffic(), "kernel": "plstm::tc::wavefront2_kernel",
            "kernel_ms": kernel_ms, "algorithmic_flops_per_launch": flops,
            "roofline_ms": roof_ms,
            "definition": "roofline time = max(FLOPs / dense peak, (T + L - 1) x probe t_step); peak = FLOPs / "
                          "roofline time; frac = roofline time / kernel time",
            "dense": {"peak": peak, "frac": achieved / peak, "floor_ms": flop_ms, "peak_note": peak_note},
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
            "clocks": clocks, "backend": model.backend_name, "parity": parity,
            "strong_scaling": strong, "configs": configs}
    print(json.dumps(line), flush=True)
    bad = [what for what, p in (("headline", parity), ("strong", (strong or {}).get("parity"))) if p and not p["ok"]]
    if bad:
        print(f"bench: parity check failed for {bad}", file=sys.stderr, flush=True)
        sys.exit(3)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-latency", action="store_true")
    ap.add_argument("--no-strong", action="store_true")
    ap.add_argument("--no-configs", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=3.0)
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
