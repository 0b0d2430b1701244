"""Benchmark of the fused B200 spectral kernels.

Default workload (the metric's single-GPU configuration, weak scaling):
signal::stft on 64 channels x 2^22 f32 samples per GPU (seeded N(0,1) plus a
linear chirp 0 -> 0.4 fs), nperseg 2048, hop 512, hann, complex64 output
(64, 1025, 8189).  A step is one call of the backend over the whole batch;
under torchrun each rank processes its own 64 channels, no collective on the
data path.

Other workloads (--workload):
  welch       one f32 channel of 2^20 samples, nperseg 1024, 50% overlap,
              hann, constant detrend, density (513 bins)
  welch_f64   1024 f64 channels x 2^20 (AR(1), phi 0.9), nperseg 4096, 50%,
              hamming, detrend 'linear' (the reference does not detrend)
  csd         512 f32 channel pairs x 2^21 given as transposed (N, C) views,
              nperseg 2048, 50%, hann, complex64 cross spectra
  coherence   the csd workload through signal::coherence (F64 Cxy)
  istft       the stft workload's complex64 output back to F64 signals
              (GSamples/s of reconstructed samples)
  welch_long  one f32 signal of 2^30 samples, nperseg 8192, 50%, blackman,
              sharded by segment range over the ranks with one NCCL
              all-reduce of the F64 partial sums (strong scaling)

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload W] [--channels C] [--no-cpu] [--no-e2e]

Rank 0 prints one JSON line.  ``value`` is input GSamples/s of all ranks
(csd counts x and y) with inputs resident in HBM, from CUDA events on the
launching stream (max over ranks); ``e2e`` is the same metric through the C
ABI with pinned host buffers, host->device copy of the inputs and
device->host copy of the result inside the timed region.  ``--impl
reference`` times the reference's own implementation (compiled from its
sources into oracle/_ref) on the host cores on a bounded sample.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "Welch/STFT input GSamples/s at 1/2/4/8 B200; % of HBM/FP32 roofline"
FP32_NOMINAL_TFLOPS = 148 * 128 * 2 * 1.965e9 / 1e12  # 74.4 (no measured FP32 peak)

WORKLOADS = {
    "stft": dict(op="stft", C=64, N=1 << 22, L=2048, H=512, window="hann",
                 dtype="f32", fs=1.0e4, desc=(
                     "signal::stft {C} ch x 2^22 f32 per GPU, nperseg 2048, hop "
                     "512, hann, complex64 out ({C}, 1025, 8189)")),
    "welch": dict(op="welch", C=1, N=1 << 20, L=1024, H=512, window="hann",
                  dtype="f32", fs=1.0e4, detrend="constant", desc=(
                      "signal::welch {C} ch x 2^20 f32 per GPU, nperseg 1024, "
                      "noverlap 512, hann, constant detrend, density")),
    "welch_f64": dict(op="welch", C=1024, N=1 << 20, L=4096, H=2048,
                      window="hamming", dtype="f64", fs=1.0, detrend="linear",
                      desc=("signal::welch f64 {C} ch x 2^20 per GPU, nperseg "
                            "4096, 50% overlap, hamming, detrend 'linear' (no "
                            "detrend, as the reference)")),
    "csd": dict(op="csd", C=512, N=1 << 21, L=2048, H=1024, window="hann",
                dtype="f32", fs=1.0, detrend="constant", desc=(
                    "signal::csd {C} f32 pairs x 2^21 per GPU as transposed "
                    "(samples, channels) views, nperseg 2048, 50%, hann, "
                    "complex64 cross spectra")),
    "coherence": dict(op="coherence", C=512, N=1 << 21, L=2048, H=1024,
                      window="hann", dtype="f32", fs=1.0, detrend="constant",
                      desc=("signal::coherence {C} f32 pairs x 2^21 per GPU as "
                            "transposed (samples, channels) views, nperseg "
                            "2048, 50%, hann (one pass over x and y)")),
    "istft": dict(op="istft", C=64, N=1 << 22, L=2048, H=512, window="hann",
                  dtype="f32", fs=1.0e4, desc=(
                      "signal::istft of the stft workload's complex64 "
                      "({C}, 1025, 8189) back to {C} ch x 4194304 F64 samples "
                      "per GPU, nperseg 2048, hop 512, hann")),
    "welch_long": dict(op="welch", C=1, N=1 << 30, L=8192, H=4096,
                       window="blackman", dtype="f32", fs=1.0, detrend="constant",
                       desc=("signal::welch one f32 signal of 2^30 samples, "
                             "nperseg 8192, noverlap 4096, blackman, segment-range "
                             "sharded over the ranks + NCCL all-reduce")),
}


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []

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
        for l in self.lines:
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
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        sm.sort()
        return {"sm_mhz": sm[len(sm) // 2], "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------
# synthetic inputs (seeded; the shapes and distributions of the workloads)
# ---------------------------------------------------------------------------
def make_inputs(torch, dev, w, rank, C):
    g = torch.Generator(device=dev)
    g.manual_seed(1000 + rank)
    N, fs = w["N"], w["fs"]
    if w["op"] in ("stft", "istft"):
        x = torch.randn((C, N), generator=g, device=dev, dtype=torch.float32)
        t = torch.arange(N, device=dev, dtype=torch.float64) / fs
        T = N / fs
        x += torch.cos(2 * math.pi * (0.5 * (0.4 * fs / T) * t * t)).float()[None, :]
        return x, None
    if w["op"] in ("csd", "coherence"):
        # x ~ N(0,1); y = 0.7 x[n-17] + 0.3 N(0,1); both as (N, C) views
        x = torch.randn((C, N), generator=g, device=dev, dtype=torch.float32)
        y = 0.7 * torch.roll(x, 17, dims=1) + 0.3 * torch.randn(
            (C, N), generator=g, device=dev, dtype=torch.float32)
        y[:, :17] = 0.3 * torch.randn((C, 17), generator=g, device=dev)
        return x.t(), y.t()
    if w["dtype"] == "f64":
        # AR(1), phi = 0.9, sigma = 1: x[n] = sum_k 0.9^k e[n-k] truncated at
        # 400 taps (0.9^400 ~ 5e-19), as a linear convolution by FFT in
        # channel chunks (input generation only)
        x = torch.empty((C, N), device=dev, dtype=torch.float64)
        K = 400
        taps = 0.9 ** torch.arange(K, device=dev, dtype=torch.float64)
        M = 1 << (N + K).bit_length()
        ft = torch.fft.rfft(taps, n=M)
        for c0 in range(0, C, 64):
            c1 = min(C, c0 + 64)
            e = torch.randn((c1 - c0, N + K - 1), generator=g, device=dev,
                            dtype=torch.float64)
            y = torch.fft.irfft(torch.fft.rfft(e, n=M) * ft, n=M)
            x[c0:c1] = y[:, K - 1:K - 1 + N]
            del e, y
        return x, None
    # f32 welch: N(0,1) + sinusoids
    if w.get("long"):
        return None, None
    x = torch.randn((C, N), generator=g, device=dev, dtype=torch.float32)
    t = torch.arange(N, device=dev, dtype=torch.float64)
    for f0 in (0.05, 0.13, 0.31):
        x += torch.sin(2 * math.pi * f0 * t).float()[None, :]
    return x, None


def make_long_span(torch, dev, w, lo, hi):
    """Samples [lo, hi) of the seeded 2^30-sample signal (N(0,1) plus 10
    sinusoids of seeded random frequency and amplitude), generated in fixed
    2^24-sample blocks so every rank sees the same global signal."""
    import numpy as np
    rng = np.random.default_rng(1005)
    freqs = rng.uniform(0.01, 0.45, 10)
    amps = rng.uniform(0.2, 2.0, 10)
    B = 1 << 24
    out = torch.empty(hi - lo, device=dev, dtype=torch.float32)
    for b0 in range((lo // B) * B, hi, B):
        g = torch.Generator(device=dev)
        g.manual_seed(5000 + b0 // B)
        blk = torch.randn(B, generator=g, device=dev, dtype=torch.float32)
        a, z = max(lo, b0), min(hi, b0 + B)
        out[a - lo:z - lo] = blk[a - b0:z - b0]
    t = torch.arange(lo, hi, device=dev, dtype=torch.float64)
    for f0, a0 in zip(freqs, amps):
        out += (a0 * torch.sin(2 * math.pi * f0 * t)).float()
    return out


# ---------------------------------------------------------------------------
# CPU baseline and the reference arm
# ---------------------------------------------------------------------------
def reference_sample(w):
    """A bounded sample of the workload for the reference on host cores."""
    import numpy as np
    rng = np.random.default_rng(2000)
    n = {"stft": 1 << 19, "welch": 1 << 20, "welch_f64": 1 << 18,
         "csd": 1 << 18, "coherence": 1 << 18, "welch_long": 1 << 21,
         "istft": 1 << 18}[w["name"]]
    x = rng.standard_normal(n)
    y = 0.7 * np.roll(x, 17) + 0.3 * rng.standard_normal(n)
    return x, y, n


def sample_units(w, n):
    """Samples one reference call on an n-sample sample accounts for."""
    if w["op"] in ("csd", "coherence"):
        return 2 * n
    if w["op"] == "istft":  # output samples of the inverse
        return ((n - w["L"]) // w["H"]) * w["H"] + w["L"]
    return n


def reference_call(w, x, y):
    """One reference call on the sample; returns (fn, kind, cores, note)."""
    from oracle import ref_runner
    cores = os.cpu_count() or 1
    L, H = w["L"], w["H"]
    if w["op"] == "istft":
        from oracle import spectral_oracle as so
        _, _, z = so.stft(x.astype("float32"), fs=w["fs"], window=w["window"],
                    nperseg=L, noverlap=L - H, complex_output=True)
    if ref_runner.available():
        kind = "reference"
        cores = ref_runner.set_threads(cores)
        if w["op"] == "istft":
            fn = lambda: ref_runner.istft(z, fs=w["fs"], window=w["window"],
                                          nperseg=L, noverlap=L - H)
            note = "reference ins::signal::istft of a one-sided complex STFT"
        elif w["op"] == "stft":
            xs = x.astype("float32")
            fn = lambda: ref_runner.stft(xs, fs=w["fs"], window=w["window"],
                                         nperseg=L, noverlap=L - H)
            note = "reference ins::signal::stft on f32"
        elif w["op"] == "csd":
            fn = lambda: ref_runner.csd(x, y, fs=w["fs"], window=w["window"],
                                        nperseg=L, noverlap=L - H)
            note = "reference ins::signal::csd on the F64-promoted pair"
        elif w["op"] == "coherence":
            fn = lambda: ref_runner.coherence(x, y, fs=w["fs"], window=w["window"],
                                              nperseg=L, noverlap=L - H)
            note = "reference ins::signal::coherence on the F64-promoted pair"
        else:
            fn = lambda: ref_runner.welch(x, fs=w["fs"], window=w["window"],
                                          nperseg=L, noverlap=L - H,
                                          detrend=w.get("detrend", "constant"))
            note = "reference ins::signal::welch on " + (
                "f64" if w["dtype"] == "f64" else "the F64-promoted signal")
    else:
        from oracle import spectral_oracle as so
        kind, cores = "port", 1
        if w["op"] == "istft":
            fn = lambda: so.istft(z, fs=w["fs"], window=w["window"], nperseg=L,
                                  noverlap=L - H)
        elif w["op"] == "stft":
            fn = lambda: so.stft(x, fs=w["fs"], window=w["window"], nperseg=L,
                                 noverlap=L - H, complex_output=True)
        elif w["op"] == "csd":
            fn = lambda: so.csd(x, y, fs=w["fs"], window=w["window"], nperseg=L,
                                noverlap=L - H)
        elif w["op"] == "coherence":
            fn = lambda: so.coherence(x, y, fs=w["fs"], window=w["window"],
                                      nperseg=L, noverlap=L - H)
        else:
            fn = lambda: so.welch(x, fs=w["fs"], window=w["window"], nperseg=L,
                                  noverlap=L - H)
        note = "numpy restatement of the reference (oracle/_ref not built)"
    return fn, kind, cores, note


def cpu_baseline(w, min_s=10.0):
    x, y, n = reference_sample(w)
    fn, kind, cores, note = reference_call(w, x, y)
    fn()
    k, t0 = 0, time.perf_counter()
    while True:
        fn()
        k += 1
        el = time.perf_counter() - t0
        if el >= min_s or k >= 100:
            break
    per = sample_units(w, n)
    gsps = k * per / el / 1e9
    seg = (n - w["L"]) // w["H"] + 1
    desc = (f"{note}, FFT by a substitute DFT for the absent FFTW3; one channel "
            f"of {n} samples ({seg} segments), {k} runs in {el:.1f} s")
    if w["op"] == "stft":
        desc += ("; its per-segment column scatter is quadratic in the segment "
                 "count, so a full 2^22-sample channel runs slower per sample")
    return {"value": gsps, "unit": "GSamples/s", "cores": cores, "kind": kind,
            "sample": desc}


def run_reference(args, w):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    x, y, n = reference_sample(w)
    fn, kind, cores, note = reference_call(w, x, y)
    for _ in range(args.warmup):
        fn()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        fn()
    el = time.perf_counter() - t0
    per = sample_units(w, n)
    v = args.steps * per / el / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": "GSamples/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": el / args.steps * 1e3, "higher_is_better": True,
        "scaling": "strong" if w["name"] == "welch_long" else "weak",
        "vs_baseline": None, "dtype": w["dtype"], "data": "synthetic",
        "config": {"workload": w["desc"].format(C=w["C"]),
                   "sample": f"{note}; one channel of {n} samples per step"},
        "cpu_baseline": {"value": v, "unit": "GSamples/s", "cores": cores,
                         "kind": kind, "sample": f"one channel of {n} samples per step"},
        "e2e": {"value": v, "unit": "GSamples/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


# ---------------------------------------------------------------------------
# our arm
# ---------------------------------------------------------------------------
def run_ours(args, w):
    import torch
    import torch.distributed as dist

    import insight_b200 as ib
    from insight_b200 import shard

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    C = args.channels or w["C"]
    L, H, op = w["L"], w["H"], w["op"]
    F = L // 2 + 1
    stream = torch.cuda.Stream(device=dev)
    kw = dict(fs=w["fs"], window=w["window"], nperseg=L, noverlap=L - H,
              stream=stream, sync=False, axes=False)
    is_long = w["name"] == "welch_long"

    if is_long:
        N = w["N"]
        s0, s1, lo, hi = shard.segment_shard(N, L, L - H, rank, world)
        x = make_long_span(torch, dev, w, lo, hi)
        y = None
        S_total = shard.framing(N, L, L - H)[1]
        samples = N  # whole signal, all ranks together
        in_bytes = (hi - lo) * 4
        out_bytes = F * 8
        nfft_work = (s1 - s0)
        def call(xin, yin, out=None):
            return shard.welch_segment_sharded(
                xin, N, rank=rank, world=world, fs=w["fs"], window=w["window"],
                nperseg=L, noverlap=L - H, detrend=w["detrend"], stream=stream)
    else:
        x, y = make_inputs(torch, dev, w, rank, C)
        N = w["N"]
        S = (N - L) // H + 1
        two = op in ("csd", "coherence")
        samples = C * N * (2 if two else 1) * world
        in_bytes = C * N * x.element_size() * (2 if two else 1)
        if op == "istft":
            # input: the stft of the seeded signal (outside the timed region)
            z = torch.empty((C, F, S), dtype=torch.complex64, device=dev)
            ib.spectral(ib.OP_STFT, x, out=z, complex_output=True,
                        **{k: v for k, v in kw.items() if k not in ("stream",)})
            torch.cuda.synchronize()
            x = z
            n_total = (S - 1) * H + L
            out = torch.empty((C, n_total), dtype=torch.float64, device=dev)
            samples = C * n_total * world
            in_bytes = C * F * S * 8
            out_bytes = C * n_total * 8
            nfft_work = C * S
            def call(xin, yin, o):
                ib.istft(xin, window=w["window"], nperseg=L, noverlap=L - H,
                         out=o, stream=stream, sync=False)
        elif op == "stft":
            out = torch.empty((C, F, S), dtype=torch.complex64, device=dev)
            out_bytes = C * F * S * 8
            nfft_work = C * S
            def call(xin, yin, o):
                ib.spectral(ib.OP_STFT, xin, out=o, complex_output=True, **kw)
        elif op == "csd":
            out = torch.empty((C, F), dtype=torch.complex64, device=dev)
            out_bytes = C * F * 8
            nfft_work = 2 * C * S
            def call(xin, yin, o):
                ib.spectral(ib.OP_CSD, xin, yin, axis=0, out=o, complex_output=True,
                            detrend=w["detrend"], **kw)
        elif op == "coherence":
            out = torch.empty((C, F), dtype=torch.float64, device=dev)
            out_bytes = C * F * 8
            nfft_work = 2 * C * S
            def call(xin, yin, o):
                ib.spectral(ib.OP_COHERENCE, xin, yin, axis=0, out=o,
                            detrend=w["detrend"], **kw)
        else:
            out = torch.empty((C, F), dtype=torch.float64, device=dev)
            out_bytes = C * F * 8
            nfft_work = C * S
            def call(xin, yin, o):
                ib.spectral(ib.OP_WELCH, xin, out=o, detrend=w["detrend"], **kw)

    run = (lambda: call(x, y)) if is_long else (lambda: call(x, y, out))
    for _ in range(args.warmup):
        run()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    launches0 = ib.launch_count()
    with ClockSampler(local) as clk:
        e0.record(stream)
        for _ in range(args.steps):
            run()
        e1.record(stream)
        torch.cuda.synchronize()
    launches = ib.launch_count() - launches0
    ms = max_over_ranks(e0.elapsed_time(e1) / args.steps)
    barrier()
    value = samples / (ms * 1e-3) / 1e9
    hbm, peak_kind = peaks()
    achieved = (in_bytes + out_bytes) / (ms * 1e-3) / 1e9
    flops = 5.0 * L * math.log2(L) * nfft_work
    fp32 = flops / (ms * 1e-3) / 1e12

    # end to end through the C ABI with pinned host buffers
    e2e = None
    if not args.no_e2e and not is_long:
        xh = (x.cpu().pin_memory() if not two
              else x.t().contiguous().cpu().pin_memory().t())
        yh = y.t().contiguous().cpu().pin_memory().t() if y is not None else None
        oh = torch.empty(out.shape, dtype=out.dtype, pin_memory=True)
        e2e_steps = max(3, min(args.steps, 10))
        for _ in range(max(1, min(args.warmup, 3))):
            call(xh, yh, oh)
        torch.cuda.synchronize()
        barrier()
        torch.cuda.synchronize()
        h0 = torch.cuda.Event(enable_timing=True)
        h1 = torch.cuda.Event(enable_timing=True)
        h0.record(stream)
        for _ in range(e2e_steps):
            call(xh, yh, oh)
        h1.record(stream)
        torch.cuda.synchronize()
        e2e_ms = max_over_ranks(h0.elapsed_time(h1) / e2e_steps)
        barrier()
        e2e = {"value": samples / (e2e_ms * 1e-3) / 1e9, "unit": "GSamples/s",
               "h2d_bytes_per_step": in_bytes, "d2h_bytes_per_step": out_bytes,
               "ms_per_step": e2e_ms}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_baseline(w)

    if rank == 0:
        config = {"workload": w["desc"].format(C=C), "samples_per_channel": w["N"],
                  "nperseg": L, "hop": H, "n_freq": F,
                  "parallelism": (f"segment-range shards x{world} + NCCL all-reduce"
                                  if is_long else f"channel shards x{world}"),
                  "l2": "inputs and outputs larger than L2 (126 MB)" if
                  in_bytes + out_bytes > (200 << 20) else
                  "input smaller than L2: L2 flushed between steps is not done"}
        if not is_long:
            config["channels_per_gpu"] = C
        line = {
            "metric": METRIC, "value": value, "unit": "GSamples/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "strong" if is_long else "weak",
            "vs_baseline": None, "dtype": w["dtype"], "data": "synthetic",
            "config": config,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm,
                         "unit": "GB/s", "frac": achieved / hbm,
                         "traffic": TRAFFIC.get(w["name"], lambda c: None)(C),
                         "peak_source": peak_kind,
                         "bytes_per_launch": in_bytes + out_bytes},
            "fp32_nominal": {"achieved_tflops": fp32, "peak_tflops":
                             FP32_NOMINAL_TFLOPS, "frac": fp32 / FP32_NOMINAL_TFLOPS,
                             "flops_per_step": flops,
                             "count": "5 nfft log2(nfft) per segment and stream"},
            "e2e": e2e,
            "cpu_baseline": cpu,
            "gpu_launches": launches,
            "clocks": clk.summary(),
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        barrier()
        dist.destroy_process_group()
    return 0


# DRAM bytes (read + write) of one launch of the dominant kernel, from the
# ncu capture summarised in profiles/ (measured on 8 channels and scaled by
# the channel count: the traffic is per channel; output bytes still in L2 at
# the end of the small capture are missing, so this is a lower bound).
TRAFFIC = {
    "stft": lambda C: (152_996_096 + 497_428_480) / 8 * C,
}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="stft", choices=sorted(WORKLOADS))
    ap.add_argument("--channels", type=int, default=0,
                    help="channels per GPU (default: the workload's)")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline")
    ap.add_argument("--no-e2e", action="store_true", help="skip the e2e leg")
    ap.add_argument("--samples", type=int, default=0,
                    help="samples per channel (default: the workload's; a "
                         "smaller case of the same kernel, for profiling)")
    args = ap.parse_args()
    w = dict(WORKLOADS[args.workload])
    w["name"] = args.workload
    if args.samples:
        w["N"] = args.samples
        w["desc"] += f" [samples per channel overridden: {args.samples}]"
    if args.impl == "reference":
        return run_reference(args, w)
    return run_ours(args, w)


if __name__ == "__main__":
    sys.exit(main())
