"""Benchmark of the fused B200 STFT (the metric's single-GPU configuration).

Workload (per GPU, weak scaling): signal::stft on 64 channels x 2^22 f32
samples (seeded N(0,1) plus a linear chirp 0 -> 0.4 fs), nperseg 2048,
hop 512 (noverlap 1536), hann window, complex64 output (64, 1025, 8189).
A step is one call of the backend over the whole batch.  Under torchrun each
rank processes its own 64-channel shard with no collective on the data path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Rank 0 prints one JSON line.  ``value`` is input GSamples/s of all ranks with
the inputs resident in HBM (max over ranks of the CUDA-event time); ``e2e``
is the same metric through the C ABI with pinned host buffers (host->device
copy of the input and device->host copy of the whole STFT inside the timed
region).  ``--impl reference`` times the reference's own stft (compiled from
its sources into oracle/_ref) on the host cores on a bounded sample.
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

CH, NSAMP, NPERSEG, NOVERLAP, FS = 64, 1 << 22, 2048, 1536, 1.0e4
METRIC = "Welch/STFT input GSamples/s at 1/2/4/8 B200; % of HBM/FP32 roofline"
WORKLOAD = ("signal::stft 64 ch x 2^22 f32, nperseg 2048, hop 512, hann, "
            "complex64 out (64, 1025, 8189) per GPU")
CPU_SAMPLE = 1 << 19  # reference stft sample: one channel prefix (1021 segments)


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def make_signal(torch, dev, seed, C=CH, N=NSAMP):
    g = torch.Generator(device=dev)
    g.manual_seed(seed)
    x = torch.randn((C, N), generator=g, device=dev, dtype=torch.float32)
    t = torch.arange(N, device=dev, dtype=torch.float64) / FS
    T = N / FS
    chirp = torch.cos(2 * torch.pi * (0.0 * t + 0.5 * (0.4 * FS / T) * t * t))
    x += chirp.to(torch.float32)[None, :]
    return x


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), "--query-gpu=" + self.Q,
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        self.lines = []
        if self.proc is not None:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()
                out = ""
            self.lines = [l for l in out.splitlines() if l.strip()]

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown",
                 "sw_power_cap"]
        for l in getattr(self, "lines", []):
            f = [v.strip() for v in l.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [],
                    "samples": 0}
        sm.sort()
        return {"sm_mhz": sm[len(sm) // 2], "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def cpu_reference_stft(x_host, reps_min_s=10.0):
    """Time the reference (oracle/_ref, else the numpy port) stft on one
    bounded sample; returns (GSamples/s, kind, cores, description)."""
    import numpy as np
    from oracle import ref_runner
    cores = os.cpu_count() or 1
    os.environ.setdefault("OMP_NUM_THREADS", str(cores))
    xs = np.ascontiguousarray(x_host[:CPU_SAMPLE], dtype=np.float32)
    if ref_runner.available():
        fn = lambda: ref_runner.stft(xs, fs=FS, window="hann", nperseg=NPERSEG,
                                     noverlap=NOVERLAP)
        kind = "reference"
    else:
        from oracle import spectral_oracle as so
        fn = lambda: so.stft(xs, fs=FS, window="hann", nperseg=NPERSEG,
                             noverlap=NOVERLAP, complex_output=True)
        kind = "port"
        cores = 1
    fn()  # warm
    n, t0 = 0, time.perf_counter()
    while True:
        fn()
        n += 1
        el = time.perf_counter() - t0
        if el >= reps_min_s or n >= 50:
            break
    gsps = n * len(xs) / el / 1e9
    desc = (f"reference ins::signal::stft (substitute DFT for the absent FFTW3) "
            f"on one f32 channel prefix of {len(xs)} samples "
            f"({(len(xs) - NPERSEG) // (NPERSEG - NOVERLAP) + 1} segments), "
            f"{n} runs in {el:.1f} s; the composite is quadratic in segments, "
            f"so a full 2^22-sample channel runs slower per sample")
    return gsps, kind, cores, desc


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    import numpy as np
    from oracle import ref_runner
    rng = np.random.default_rng(1002)
    n = CPU_SAMPLE
    t = np.arange(n) / FS
    x = (rng.standard_normal(n) + np.cos(
        2 * np.pi * 0.5 * (0.4 * FS / (NSAMP / FS)) * t * t)).astype(np.float32)
    cores = os.cpu_count() or 1
    if ref_runner.available():
        fn = lambda: ref_runner.stft(x, fs=FS, window="hann", nperseg=NPERSEG,
                                     noverlap=NOVERLAP)
        kind = "reference"
    else:
        from oracle import spectral_oracle as so
        fn = lambda: so.stft(x, fs=FS, window="hann", nperseg=NPERSEG,
                             noverlap=NOVERLAP, complex_output=True)
        kind, cores = "port", 1
    for _ in range(args.warmup):
        fn()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        fn()
    el = time.perf_counter() - t0
    v = args.steps * n / el / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": "GSamples/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": el / args.steps * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": WORKLOAD, "sample": f"one channel prefix, {n} samples",
                   "l2": "host run"},
        "cpu_baseline": {"value": v, "unit": "GSamples/s", "cores": cores,
                         "kind": kind,
                         "sample": f"one f32 channel prefix of {n} samples per step"},
        "e2e": {"value": v, "unit": "GSamples/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_ours(args):
    import torch
    import torch.distributed as dist

    import insight_b200 as ib

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                device_id=dev)

    x = make_signal(torch, dev, 1002 + rank)
    C, N = x.shape
    F = NPERSEG // 2 + 1
    S = (N - NPERSEG) // (NPERSEG - NOVERLAP) + 1
    out = torch.empty((C, F, S), dtype=torch.complex64, device=dev)
    stream = torch.cuda.Stream(device=dev)
    call = lambda xin, o: ib.spectral(
        ib.OP_STFT, xin, fs=FS, window="hann", nperseg=NPERSEG, noverlap=NOVERLAP,
        complex_output=True, out=o, stream=stream, sync=False, axes=False)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    # device-resident timing
    for _ in range(args.warmup):
        call(x, out)
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    launches0 = ib.launch_count()
    with ClockSampler(local) as clk:
        e0.record(stream)
        for _ in range(args.steps):
            call(x, out)
        e1.record(stream)
        torch.cuda.synchronize()
    launches = ib.launch_count() - launches0
    ms = e0.elapsed_time(e1) / args.steps
    barrier()
    ms = max_over_ranks(ms)
    samples = C * N
    value = world * samples / (ms * 1e-3) / 1e9
    in_bytes = samples * 4
    out_bytes = C * F * S * 8
    hbm, peak_kind = peaks()
    achieved = (in_bytes + out_bytes) / (ms * 1e-3) / 1e9

    # end to end through the C ABI with pinned host buffers
    xh = x.cpu().pin_memory()
    oh = torch.empty((C, F, S), dtype=torch.complex64, pin_memory=True)
    e2e_steps = max(3, min(args.steps, 10))
    for _ in range(max(1, min(args.warmup, 3))):
        call(xh, oh)
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    h0 = torch.cuda.Event(enable_timing=True)
    h1 = torch.cuda.Event(enable_timing=True)
    h0.record(stream)
    for _ in range(e2e_steps):
        call(xh, oh)
    h1.record(stream)
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(h0.elapsed_time(h1) / e2e_steps)
    barrier()
    e2e = world * samples / (e2e_ms * 1e-3) / 1e9
    ok = bool(torch.isfinite(torch.view_as_real(oh[0, :, :4])).all())

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        v, kind, cores, desc = cpu_reference_stft(xh[0].numpy())
        cpu = {"value": v, "unit": "GSamples/s", "cores": cores, "kind": kind,
               "sample": desc}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": "GSamples/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic",
            "config": {"workload": WORKLOAD, "channels_per_gpu": C,
                       "samples_per_channel": N, "nperseg": NPERSEG,
                       "hop": NPERSEG - NOVERLAP, "n_freq": F, "n_seg": S,
                       "output": "complex64 (C, F, S)", "parallelism": f"channel shards x{world}",
                       "l2": "inputs (1 GiB) and outputs (4.3 GB) larger than L2"},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm,
                         "unit": "GB/s", "frac": achieved / hbm, "traffic": None,
                         "peak_source": peak_kind,
                         "bytes_per_launch": in_bytes + out_bytes},
            "e2e": {"value": e2e, "unit": "GSamples/s",
                    "h2d_bytes_per_step": in_bytes, "d2h_bytes_per_step": out_bytes,
                    "ms_per_step": e2e_ms, "finite": ok},
            "cpu_baseline": cpu,
            "gpu_launches": launches,
            "clocks": clk.summary(),
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        barrier()
        dist.destroy_process_group()
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu", action="store_true",
                    help="skip the CPU baseline leg")
    args = ap.parse_args()
    if args.impl == "reference":
        return run_reference(args)
    return run_ours(args)


if __name__ == "__main__":
    sys.exit(main())
