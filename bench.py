"""Benchmark of the fused B200 spectral kernels.

Default workload (the metric's single-GPU configuration): signal::stft on 64
channels x 2^22 f32 samples (seeded N(0,1) plus a linear chirp 0 -> 0.4 fs),
nperseg 2048, hop 512, hann, complex64 output (64, 1025, 8189).  A step is
one call of the backend over this rank's channels; under torchrun the 64
channels are split into contiguous blocks over the ranks (strong scaling: the
total work is the workload's), with no collective on the data path.

The same run also measures, device-resident and with the same step count,
the other workloads ("workloads" in the JSON line):
  welch       one f32 channel of 2^20 samples, nperseg 1024, 50% overlap,
              hann, constant detrend, density (513 bins); one replica per
              rank when there are more ranks than channels
  welch_f64   1024 f64 channels x 2^20 (AR(1), phi 0.9), nperseg 4096, 50%,
              hamming, detrend 'linear' (the reference does not detrend),
              channel-sharded
  csd         512 f32 channel pairs x 2^21 given as transposed (N, C) views,
              nperseg 2048, 50%, hann, complex64 cross spectra, pair-sharded
  coherence   the csd workload through signal::coherence (F64 Cxy)
  istft       the stft workload's complex64 output back to F64 signals
              (GSamples/s of reconstructed samples), channel-sharded
  welch_long  one f32 signal of 2^30 samples, nperseg 8192, 50%, blackman,
              sharded by segment range over the ranks: each rank's F64
              partial PSD (its segments, averaged with the whole signal's
              segment count) and one NCCL all-reduce per step; a step
              replays the rank's kernels as a captured CUDA graph, and the
              regular call is timed beside it; the line carries each rank's
              partial / all-reduce times (finalize: no work after the
              all-reduce)

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload W] [--channels C] [--samples N] [--no-cpu]
                    [--no-e2e] [--no-extra]

Rank 0 prints one JSON line.  ``value`` is input GSamples/s of all ranks
(csd counts x and y) with inputs resident in HBM, from CUDA events on the
launching stream (max over ranks); ``e2e`` is the same metric through the
public API with pinned host buffers, host->device copy of the inputs and
device->host copy of the result inside the timed region.  ``--impl
reference`` times the reference's own implementation (compiled from its
sources into oracle/_ref) on the host cores on a bounded sample.
--workload, --channels or --samples measure that one workload only.
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
                     "signal::stft {C} ch x 2^22 f32, nperseg 2048, hop 512, "
                     "hann, complex64 out ({C}, 1025, 8189)")),
    "welch": dict(op="welch", C=1, N=1 << 20, L=1024, H=512, window="hann",
                  dtype="f32", fs=1.0e4, detrend="constant", plan=True, desc=(
                      "signal::welch {C} ch x 2^20 f32, nperseg 1024, "
                      "noverlap 512, hann, constant detrend, density")),
    "welch_f64": dict(op="welch", C=1024, N=1 << 20, L=4096, H=2048,
                      window="hamming", dtype="f64", fs=1.0, detrend="linear",
                      desc=("signal::welch f64 {C} ch x 2^20, nperseg "
                            "4096, 50% overlap, hamming, detrend 'linear' (no "
                            "detrend, as the reference)")),
    "csd": dict(op="csd", C=512, N=1 << 21, L=2048, H=1024, window="hann",
                dtype="f32", fs=1.0, detrend="constant", desc=(
                    "signal::csd {C} f32 pairs x 2^21 as transposed "
                    "(samples, channels) views, nperseg 2048, 50%, hann, "
                    "complex64 cross spectra")),
    "coherence": dict(op="coherence", C=512, N=1 << 21, L=2048, H=1024,
                      window="hann", dtype="f32", fs=1.0, detrend="constant",
                      desc=("signal::coherence {C} f32 pairs x 2^21 as "
                            "transposed (samples, channels) views, nperseg "
                            "2048, 50%, hann (one pass over x and y)")),
    "istft": dict(op="istft", C=64, N=1 << 22, L=2048, H=512, window="hann",
                  dtype="f32", fs=1.0e4, desc=(
                      "signal::istft of the stft workload's complex64 "
                      "({C}, 1025, 8189) back to {C} ch x 4194304 F64 samples, "
                      "nperseg 2048, hop 512, hann")),
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
def make_inputs(torch, dev, w, c0, C):
    """Channels [c0, c0 + C) of the workload's seeded input."""
    g = torch.Generator(device=dev)
    g.manual_seed(1000 + c0)
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
    desc = (f"{note}, FFT by a substitute radix-2 FFT for the absent FFTW3; one channel "
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
        "scaling": "strong",
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
class Ranks:
    """One process per GPU: barrier, max over ranks and an all-ranks flag."""

    def __init__(self, torch, world, rank, local, dev):
        self.torch, self.world, self.rank, self.local, self.dev = (
            torch, world, rank, local, dev)
        if world > 1:
            import torch.distributed as dist
            self.dist = dist

    def barrier(self):
        if self.world > 1:
            self.dist.barrier(device_ids=[self.local])

    def max(self, v):
        if self.world == 1:
            return v
        t = self.torch.tensor([v], dtype=self.torch.float64, device=self.dev)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def all_ok(self, ok):
        if self.world == 1:
            return ok
        t = self.torch.tensor([1.0 if ok else 0.0], dtype=self.torch.float64,
                              device=self.dev)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MIN)
        return t.item() > 0.5

    def gather_rows(self, row):
        """[world, len(row)] table of every rank's row (on every rank)."""
        t = self.torch.zeros((self.world, len(row)), dtype=self.torch.float64,
                             device=self.dev)
        t[self.rank] = self.torch.tensor(row, dtype=self.torch.float64)
        if self.world > 1:
            self.dist.all_reduce(t)
        return t.cpu().tolist()


def setup(torch, w, dev, rank, world, stream):
    """This rank's share of the workload, resident in HBM, and a one-step
    callable.  Channel batches split the workload's channels into contiguous
    blocks (strong scaling: the total is the workload's); the long signal is
    split by segment range with one NCCL all-reduce per step; a workload with
    fewer channels than ranks runs one replica per rank."""
    import insight_b200 as ib
    from insight_b200 import shard

    L, H, op = w["L"], w["H"], w["op"]
    F = L // 2 + 1
    kw = dict(fs=w["fs"], window=w["window"], nperseg=L, noverlap=L - H,
              stream=stream, sync=False, axes=False)
    st = {"F": F, "L": L}
    if w["name"] == "welch_long":
        N = w["N"]
        s0, s1, lo, hi = shard.segment_shard(N, L, L - H, rank, world)
        x = make_long_span(torch, dev, w, lo, hi)

        def call_step(on_phase=None):
            return shard.welch_segment_sharded(
                x, N, rank=rank, world=world, fs=w["fs"], window=w["window"],
                nperseg=L, noverlap=L - H, detrend=w["detrend"], stream=stream,
                on_phase=on_phase)
        # the same step with this rank's kernels captured once into a CUDA
        # graph (the span tensor is fixed); the regular call is timed beside it
        plan = shard.SegmentShardPlan(
            x, N, rank=rank, world=world, fs=w["fs"], window=w["window"],
            nperseg=L, noverlap=L - H, detrend=w["detrend"], stream=stream)
        step = lambda on_phase=None: plan.run(on_phase=on_phase)
        st.update(plan=plan, call_step=call_step)
        st.update(step=step, samples_total=N, in_bytes=(hi - lo) * 4,
                  out_bytes=F * 8, transforms=s1 - s0, C_local=1,
                  parallelism=(f"segment-range shards x{world} + one NCCL "
                               "all-reduce of F f64 partial sums per step"
                               if world > 1 else "one GPU"),
                  scaling="strong", detail={"segments_per_rank": s1 - s0,
                                            "halo_samples": L - H})
        return st

    C_total = w["C"]
    if C_total >= world:
        c0, c1 = shard.block_range(C_total, rank, world)
        scaling = "strong"
        par = f"channel shards x{world}, no collective" if world > 1 else "one GPU"
        C_all = C_total  # channels processed by all ranks together
    else:
        c0, c1 = 0, C_total
        scaling = "weak"
        par = f"replicas x{world} (fewer channels than GPUs)"
        C_all = C_total * world
    C = c1 - c0
    x, y = make_inputs(torch, dev, w, c0, C)
    N = w["N"]
    S = (N - L) // H + 1
    two = op in ("csd", "coherence")
    in_bytes = C * N * x.element_size() * (2 if two else 1)
    samples_total = C_all * N * (2 if two else 1)
    if op == "istft":
        z = torch.empty((C, F, S), dtype=torch.complex64, device=dev)
        ib.spectral(ib.OP_STFT, x, out=z, complex_output=True,
                    **{k: v for k, v in kw.items() if k != "stream"})
        torch.cuda.synchronize()
        del x
        x = z
        n_total = (S - 1) * H + L
        out = torch.empty((C, n_total), dtype=torch.float64, device=dev)
        samples_total = C_all * n_total
        in_bytes = C * F * S * 8
        out_bytes = C * n_total * 8
        transforms = C * S

        def call(xin, yin, o):
            ib.istft(xin, window=w["window"], nperseg=L, noverlap=L - H, out=o,
                     stream=stream, sync=False)
    elif op == "stft":
        out = torch.empty((C, F, S), dtype=torch.complex64, device=dev)
        out_bytes = C * F * S * 8
        transforms = C * S

        def call(xin, yin, o):
            ib.spectral(ib.OP_STFT, xin, out=o, complex_output=True, **kw)
    elif op == "csd":
        out = torch.empty((C, F), dtype=torch.complex64, device=dev)
        out_bytes = C * F * 8
        transforms = 2 * C * S

        def call(xin, yin, o):
            ib.spectral(ib.OP_CSD, xin, yin, axis=0, out=o, complex_output=True,
                        detrend=w["detrend"], **kw)
    elif op == "coherence":
        out = torch.empty((C, F), dtype=torch.float64, device=dev)
        out_bytes = C * F * 8
        transforms = 2 * C * S

        def call(xin, yin, o):
            ib.spectral(ib.OP_COHERENCE, xin, yin, axis=0, out=o,
                        detrend=w["detrend"], **kw)
    else:
        out = torch.empty((C, F), dtype=torch.float64, device=dev)
        out_bytes = C * F * 8
        transforms = C * S

        def call(xin, yin, o):
            ib.spectral(ib.OP_WELCH, xin, out=o, detrend=w["detrend"], **kw)
    step = lambda on_phase=None: call(x, y, out)
    if w.get("plan"):
        # a short signal: the call is bound by host work and launch latency,
        # so the step replays it as a captured CUDA graph (SpectralPlan); the
        # regular call is timed beside it
        plan = ib.SpectralPlan(
            ib.OP_WELCH, x, out=out, detrend=w["detrend"],
            **{k: v for k, v in kw.items() if k not in ("sync", "axes")})
        st["plan"] = plan
        st["call_step"] = step
        step = lambda on_phase=None: plan.run(stream=stream)
    st.update(step=step, call=call, x=x, y=y,
              out=out, two=two, samples_total=samples_total, in_bytes=in_bytes,
              out_bytes=out_bytes, transforms=transforms, C_local=C,
              parallelism=par, scaling=scaling, detail={"channels_per_gpu": C})
    return st


def timed(torch, R, stream, step, steps, warmup):
    """W warm-up steps, then K steps between CUDA events on the launching
    stream, bracketed by barrier + synchronize; the max over ranks."""
    import insight_b200 as ib
    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    R.barrier()
    torch.cuda.synchronize()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    launches0 = ib.launch_count()
    with ClockSampler(R.local) as clk:
        e0.record(stream)
        h0 = time.perf_counter()
        for _ in range(steps):
            step()
        h1 = time.perf_counter()
        e1.record(stream)
        torch.cuda.synchronize()
    launches = ib.launch_count() - launches0
    ms_local = e0.elapsed_time(e1) / steps
    ms = R.max(ms_local)
    R.barrier()
    clocks = clk.summary()
    # host time to enqueue one step (a step whose device time is not much
    # above this is bound by the host, not by the kernels)
    clocks["host_enqueue_ms_per_step"] = (h1 - h0) * 1e3 / steps
    return ms, ms_local, launches, clocks


def phase_breakdown(torch, R, stream, step, steps):
    """Per-rank device time of the long welch's three steps (partial sums,
    all-reduce, finalize), from events recorded on the launching stream
    between them, averaged over `steps` steps."""
    names = ("partial", "all_reduce", "finalize")
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(4)]
          for _ in range(steps)]
    torch.cuda.synchronize()
    R.barrier()
    torch.cuda.synchronize()
    for k in range(steps):
        e = ev[k]
        e[0].record(stream)
        step(on_phase=lambda name, e=e: e[1 + names.index(name)].record(stream))
    torch.cuda.synchronize()
    row = [sum(ev[k][i].elapsed_time(ev[k][i + 1]) for k in range(steps)) / steps
           for i in range(3)]
    table = R.gather_rows(row)
    R.barrier()
    return {"unit": "ms per step (CUDA events on the launching stream)",
            "per_rank": [dict(zip(names, r)) for r in table],
            "max_over_ranks": {n: max(r[i] for r in table)
                               for i, n in enumerate(names)}}


def roofline_of(w, st, ms):
    """Algorithmic bytes and nominal FLOPs of one step of this rank against
    the measured HBM copy peak and the nominal FP32 / FP64 rates; the bound is
    whichever takes longer."""
    hbm, peak_kind = peaks()
    byts = st["in_bytes"] + st["out_bytes"]
    flops = 5.0 * st["L"] * math.log2(st["L"]) * st["transforms"]
    fp_peak = FP32_NOMINAL_TFLOPS / (2 if w["dtype"] == "f64" else 1)
    t_hbm = byts / (hbm * 1e9)
    t_fp = flops / (fp_peak * 1e12)
    r = {"bytes_per_launch": byts, "flops_per_step": flops,
         "hbm": {"achieved": byts / (ms * 1e-3) / 1e9, "peak": hbm,
                 "unit": "GB/s", "frac": t_hbm / (ms * 1e-3),
                 "peak_source": peak_kind},
         "fp": {"achieved": flops / (ms * 1e-3) / 1e12, "peak": fp_peak,
                "unit": "TFLOP/s", "frac": t_fp / (ms * 1e-3),
                "peak_source": "nominal (%s: 148 SMs x 128 lanes x 2 x 1.965 GHz%s)"
                % ("FP64" if w["dtype"] == "f64" else "FP32",
                   ", halved" if w["dtype"] == "f64" else ""),
                "count": "5 nfft log2(nfft) per transformed segment and stream"}}
    r["bound"] = "hbm" if t_hbm >= t_fp else ("fp64" if w["dtype"] == "f64" else "fp32")
    r["frac"] = max(t_hbm, t_fp) / (ms * 1e-3)
    return r


def measure_extra(torch, R, name, dev, stream, steps, warmup):
    """One more workload measured in the same run (device-resident inputs)."""
    w = dict(WORKLOADS[name])
    w["name"] = name
    st, err = None, None
    try:
        st = setup(torch, w, dev, R.rank, R.world, stream)
        st["step"]()
        torch.cuda.synchronize()
    except Exception as e:  # recorded in the line; every rank skips together
        err = f"{type(e).__name__}: {e}"
    if not R.all_ok(err is None):
        st = None
        torch.cuda.empty_cache()
        return {"error": err or "failed on another rank"}
    ms, ms_local, launches, clocks = timed(torch, R, stream, st["step"], steps,
                                           warmup)
    res = {"workload": w["desc"].format(C=w["C"]), "dtype": w["dtype"],
           "value": st["samples_total"] / (ms * 1e-3) / 1e9, "unit": "GSamples/s",
           "ms_per_step": ms, "steps": steps, "warmup": warmup,
           "scaling": st["scaling"], "parallelism": st["parallelism"],
           "gpu_launches": launches, "clocks": clocks,
           "roofline": roofline_of(w, st, ms_local)}
    res.update(st["detail"])
    if "call_step" in st:
        cms, _, _, cclk = timed(torch, R, stream, st["call_step"], steps, warmup)
        res["plan"] = ("value and ms_per_step replay this rank's kernels as a "
                       "captured CUDA graph (SpectralPlan); ms_per_step_call is "
                       "the regular call")
        res["ms_per_step_call"] = cms
        res["host_enqueue_ms_per_step_call"] = cclk["host_enqueue_ms_per_step"]
    if name == "welch_long":
        res["breakdown"] = phase_breakdown(torch, R, stream, st["step"], steps)
        res["breakdown_call"] = phase_breakdown(torch, R, stream, st["call_step"],
                                                steps)
    if "plan" in st:
        st["plan"].close()
    del st
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    return res


EXTRAS = ("welch", "welch_f64", "csd", "coherence", "istft", "welch_long")


def run_ours(args, w):
    import torch

    import insight_b200 as ib  # noqa: F401  (fails loudly without the backend)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import torch.distributed as dist
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                device_id=dev)
    R = Ranks(torch, world, rank, local, dev)
    stream = torch.cuda.Stream(device=dev)

    st = setup(torch, w, dev, rank, world, stream)
    ms, ms_local, launches, clocks = timed(torch, R, stream, st["step"],
                                           args.steps, args.warmup)
    value = st["samples_total"] / (ms * 1e-3) / 1e9
    roof = roofline_of(w, st, ms_local)
    breakdown = breakdown_call = None
    if w["name"] == "welch_long":
        breakdown = phase_breakdown(torch, R, stream, st["step"], args.steps)
        breakdown_call = phase_breakdown(torch, R, stream, st["call_step"],
                                         args.steps)
    call_ms = call_host = None
    if "call_step" in st:
        call_ms, _, _, cclk = timed(torch, R, stream, st["call_step"], args.steps,
                                    args.warmup)
        call_host = cclk["host_enqueue_ms_per_step"]

    # end to end through the public API with pinned host buffers
    e2e = None
    if not args.no_e2e and "call" in st:
        x, y, out, call = st["x"], st["y"], st["out"], st["call"]
        xh = (x.cpu().pin_memory() if not st["two"]
              else x.t().contiguous().cpu().pin_memory().t())
        yh = y.t().contiguous().cpu().pin_memory().t() if y is not None else None
        oh = torch.empty(out.shape, dtype=out.dtype, pin_memory=True)
        e2e_steps = max(3, min(args.steps, 10))
        e2e_ms, _, _, _ = timed(torch, R, stream, lambda: call(xh, yh, oh),
                                e2e_steps, max(1, min(args.warmup, 3)))
        e2e = {"value": st["samples_total"] / (e2e_ms * 1e-3) / 1e9,
               "unit": "GSamples/s", "h2d_bytes_per_step": st["in_bytes"],
               "d2h_bytes_per_step": st["out_bytes"], "ms_per_step": e2e_ms,
               "note": ("per GPU: pinned host input copied in and the whole "
                        "result copied out every step, in channel chunks that "
                        "overlap the copies with the kernels; bound by the "
                        "host<->device copies (PCIe, and the host memory that "
                        "all GPUs of the node share), not by the kernels")}
        del xh, yh, oh
    if "plan" in st:
        st.pop("plan").close()
    for k in ("x", "y", "out", "step", "call", "call_step"):
        st.pop(k, None)
    torch.cuda.synchronize()
    torch.cuda.empty_cache()

    extras = {}
    if not args.no_extra:
        for name in EXTRAS:
            if name != w["name"]:
                extras[name] = measure_extra(torch, R, name, dev, stream,
                                             args.steps, args.warmup)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_baseline(w)

    if rank == 0:
        C = w["C"]
        in_b, out_b = st["in_bytes"], st["out_bytes"]
        config = {"workload": w["desc"].format(C=C), "samples_per_channel": w["N"],
                  "nperseg": st["L"], "hop": w["H"], "n_freq": st["F"],
                  "parallelism": st["parallelism"],
                  "l2": "inputs and outputs larger than L2 (126 MB)" if
                  in_b + out_b > (200 << 20) else
                  "input smaller than L2: L2 flushed between steps is not done"}
        config.update(st["detail"])
        line = {
            "metric": METRIC, "value": value, "unit": "GSamples/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": st["scaling"],
            "vs_baseline": None, "dtype": w["dtype"], "data": "synthetic",
            "config": config,
            "roofline": {"bound": "hbm", "achieved": roof["hbm"]["achieved"],
                         "peak": roof["hbm"]["peak"], "unit": "GB/s",
                         "frac": roof["hbm"]["frac"],
                         "traffic": TRAFFIC.get(w["name"], lambda c: None)(
                             st["C_local"]),
                         "peak_source": roof["hbm"]["peak_source"],
                         "bytes_per_launch": in_b + out_b,
                         "kernel_ms": ms_local},
            "fp_nominal": roof["fp"],
            "e2e": e2e,
            "cpu_baseline": cpu,
            "gpu_launches": launches,
            "clocks": clocks,
        }
        if breakdown is not None:
            line["breakdown"] = breakdown
            line["breakdown_call"] = breakdown_call
        if call_ms is not None:
            line["plan"] = ("value and ms_per_step replay this rank's kernels as "
                            "a captured CUDA graph (SpectralPlan); "
                            "ms_per_step_call is the regular call")
            line["ms_per_step_call"] = call_ms
            line["host_enqueue_ms_per_step_call"] = call_host
        if extras:
            line["workloads"] = extras
        print(json.dumps(line), flush=True)
    if world > 1:
        R.barrier()
        import torch.distributed as dist
        dist.destroy_process_group()
    return 0


# DRAM bytes (read + write) of one launch of the dominant kernel, from the
# ncu capture summarised in profiles/ (measured on 8 channels and scaled by
# the channel count: the traffic is per channel; output bytes still in L2 at
# the end of the small capture are missing, so this is a lower bound).
TRAFFIC = {
    "stft": lambda C: (140_656_384 + 489_337_856) / 8 * C,
}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="stft", choices=sorted(WORKLOADS))
    ap.add_argument("--channels", type=int, default=0,
                    help="channels in all (default: the workload's)")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline")
    ap.add_argument("--no-e2e", action="store_true", help="skip the e2e leg")
    ap.add_argument("--no-extra", action="store_true",
                    help="measure the selected workload only")
    ap.add_argument("--samples", type=int, default=0,
                    help="samples per channel (default: the workload's; a "
                         "smaller case of the same kernel, for profiling)")
    args = ap.parse_args()
    w = dict(WORKLOADS[args.workload])
    w["name"] = args.workload
    if args.workload != "stft" or args.channels or args.samples:
        args.no_extra = True
    if args.channels:
        w["C"] = args.channels
    if args.samples:
        w["N"] = args.samples
        w["desc"] += f" [samples per channel overridden: {args.samples}]"
    if args.impl == "reference":
        return run_reference(args, w)
    return run_ours(args, w)


if __name__ == "__main__":
    sys.exit(main())
