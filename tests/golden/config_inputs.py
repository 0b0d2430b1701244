"""Seeded inputs of the benchmark configurations, one channel (or pair) each.

Shared by tests/golden/make_config_golden.py, which runs the reference on
them and commits only the reference's outputs (reference_configs.npz), and by
the tests, which regenerate the same inputs from the same seeds with numpy's
PCG64 generator instead of loading megabytes of samples.

  config_1  welch: one f32 channel of 2^20 samples, N(0,1) plus unit sinusoids
            at 0.05, 0.13 and 0.31 fs; fs 1e4, nperseg 1024, noverlap 512,
            hann, constant detrend, density
  config_2  stft: f32 N(0,1) plus a linear chirp 0 -> 0.4 fs; nperseg 2048,
            hop 512, hann; one segment (2048 samples) and eight segments
            (5632 samples)
  config_3  welch f64: one AR(1) channel (phi 0.9, sigma 1) of 2^20 samples;
            nperseg 4096, 50%, hamming, detrend 'linear' (no detrend in the
            reference)
  config_4  csd: one f32 pair of 2^21 samples, x ~ N(0,1),
            y = 0.7 x[n-17] + 0.3 N(0,1); nperseg 2048, 50%, hann
  config_5  welch: the first 2^21 samples of an f32 signal of N(0,1) plus 10
            sinusoids of seeded random frequency and amplitude; nperseg 8192,
            noverlap 4096, blackman
"""
from __future__ import annotations

import numpy as np


def config_1():
    rng = np.random.default_rng(3001)
    n = 1 << 20
    t = np.arange(n, dtype=np.float64)
    x = rng.standard_normal(n)
    for f0 in (0.05, 0.13, 0.31):
        x = x + np.sin(2 * np.pi * f0 * t)
    return x.astype(np.float32)


def config_2(n):
    rng = np.random.default_rng(3002)
    fs = 1.0e4
    t = np.arange(n, dtype=np.float64) / fs
    T = n / fs
    x = rng.standard_normal(n) + np.cos(2 * np.pi * (0.5 * (0.4 * fs / T) * t * t))
    return x.astype(np.float32)


def config_3():
    rng = np.random.default_rng(3003)
    n = 1 << 20
    e = rng.standard_normal(n + 400)
    # x[n] = 0.9 x[n-1] + e[n], started 400 samples early (0.9^400 ~ 5e-19)
    from scipy.signal import lfilter
    return lfilter([1.0], [1.0, -0.9], e)[400:].astype(np.float64)


def config_4():
    rng = np.random.default_rng(3004)
    n = 1 << 21
    x = rng.standard_normal(n)
    y = 0.7 * np.concatenate([np.zeros(17), x[:-17]]) + 0.3 * rng.standard_normal(n)
    return x.astype(np.float32), y.astype(np.float32)


def config_5():
    rng = np.random.default_rng(3005)
    n = 1 << 21
    freqs = rng.uniform(0.01, 0.45, 10)
    amps = rng.uniform(0.2, 2.0, 10)
    t = np.arange(n, dtype=np.float64)
    x = rng.standard_normal(n)
    for f0, a0 in zip(freqs, amps):
        x = x + a0 * np.sin(2 * np.pi * f0 * t)
    return x.astype(np.float32)


# (name, input function, op, kwargs of the call)
CASES = [
    ("config_1", config_1, "welch",
     dict(fs=1.0e4, window="hann", nperseg=1024, noverlap=512,
          detrend="constant")),
    ("config_2_one_segment", lambda: config_2(2048), "stft",
     dict(fs=1.0e4, window="hann", nperseg=2048, noverlap=1536)),
    ("config_2_eight_segments", lambda: config_2(2048 + 7 * 512), "stft",
     dict(fs=1.0e4, window="hann", nperseg=2048, noverlap=1536)),
    ("config_3", config_3, "welch",
     dict(fs=1.0, window="hamming", nperseg=4096, noverlap=2048,
          detrend="linear")),
    ("config_4", config_4, "csd",
     dict(fs=1.0, window="hann", nperseg=2048, noverlap=1024,
          detrend="constant")),
    ("config_5", config_5, "welch",
     dict(fs=1.0, window="blackman", nperseg=8192, noverlap=4096,
          detrend="constant")),
]
