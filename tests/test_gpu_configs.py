"""The CUDA path against the reference's own outputs at the benchmark
configurations' parameters (tests/golden/reference_configs.npz, made by
tests/golden/make_config_golden.py from one channel or pair of each
configuration's seeded input).

Each case runs the shapes the benchmarks run: the f32 stft at nperseg 2048 /
hop 512 through the warp-specialised complex kernel and the reference's F64
Re(X) layout, the f64 welch at 4096 with hamming and detrend 'linear', the
csd pair as one column of a transposed (samples, channels) view, and the
long-signal welch at 8192 with blackman, whole and as segment-range shards
reduced on the host.  Parity bar: f and t bit-exact, max |got - ref| /
max |ref| <= 1e-5 for f32 inputs (computed in f32 against the reference's
F64-promoted result) and <= 1e-12 for f64.
"""
import os
import sys

import numpy as np
import pytest

import insight_b200 as ib
from insight_b200 import shard
from oracle import spectral_oracle as so

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
sys.path.insert(0, GOLDEN)
import config_inputs as ci  # noqa: E402

CASES = {c[0]: c for c in ci.CASES}


@pytest.fixture(scope="module")
def g():
    return np.load(os.path.join(GOLDEN, "reference_configs.npz"))


def _np(a):
    return a.detach().cpu().numpy() if hasattr(a, "detach") else np.asarray(a)


def test_config_1_welch(g, cuda):
    import torch
    _, make, _, kw = CASES["config_1"]
    x = torch.from_numpy(make()).to(cuda)
    r = ib.welch(x, **kw)
    assert np.array_equal(_np(r.f), g["config_1/f"])
    assert so.max_rel_err(_np(r.Pxx), g["config_1/Pxx"]) <= 1e-5
    # the native batched entry on the same channel (device-resident result)
    _, p = ib.spectral(ib.OP_WELCH, x[None, :], **kw)
    assert so.max_rel_err(_np(p)[0], g["config_1/Pxx"]) <= 1e-5


@pytest.mark.parametrize("name", ["config_2_one_segment", "config_2_eight_segments"])
def test_config_2_stft(name, g, cuda):
    import torch
    _, make, _, kw = CASES[name]
    xh = make()
    x = torch.from_numpy(xh).to(cuda)
    nfft = kw["nperseg"]
    # reference-signature stft: Re(X) as F64 (n_seg, n_freq)
    r = ib.stft(x, **kw)
    assert np.array_equal(_np(r.f), g[name + "/f"])
    assert np.array_equal(_np(r.t), g[name + "/t"])
    got = so.reference_spectrogram_layout(_np(r.Sxx), "complex", nfft)
    assert so.max_rel_err(got, g[name + "/Sxx"]) <= 1e-5
    # complex64 (F, S) through the warp-specialised kernel, in a batch of 4
    # channels so whole tiles of segment pairs run; this channel is number 2
    rng = np.random.default_rng(5)
    xb = np.stack([rng.standard_normal(len(xh)).astype(np.float32) for _ in range(4)])
    xb[2] = xh
    _, _, z = ib.spectral(ib.OP_STFT, torch.from_numpy(xb).to(cuda),
                          complex_output=True, **kw)
    zr = _np(z)[2].real.T
    got = so.reference_spectrogram_layout(zr, "complex", nfft)
    assert so.max_rel_err(got, g[name + "/Sxx"]) <= 1e-5
    if zr.shape[0] == 1:  # one segment: the reference writes every bin
        assert so.max_rel_err(zr, g[name + "/Sxx"]) <= 1e-5


def test_config_3_welch_f64(g, cuda):
    import torch
    _, make, _, kw = CASES["config_3"]
    xh = make()
    r = ib.welch(torch.from_numpy(xh).to(cuda), **kw)
    assert np.array_equal(_np(r.f), g["config_3/f"])
    assert so.max_rel_err(_np(r.Pxx), g["config_3/Pxx"]) <= 1e-12
    # as channel 1 of a 3-channel batch (the batched accumulate kernel)
    rng = np.random.default_rng(6)
    xb = np.stack([rng.standard_normal(len(xh)), xh, rng.standard_normal(len(xh))])
    _, p = ib.spectral(ib.OP_WELCH, torch.from_numpy(xb).to(cuda), **kw)
    assert so.max_rel_err(_np(p)[1], g["config_3/Pxx"]) <= 1e-12


def test_config_4_csd_transposed_view(g, cuda):
    import torch
    _, make, _, kw = CASES["config_4"]
    xh, yh = make()
    rng = np.random.default_rng(7)
    X = np.stack([rng.standard_normal(len(xh)).astype(np.float32), xh,
                  rng.standard_normal(len(xh)).astype(np.float32)])
    Y = np.stack([rng.standard_normal(len(yh)).astype(np.float32), yh,
                  rng.standard_normal(len(yh)).astype(np.float32)])
    xt = torch.from_numpy(X).to(cuda).t()  # (samples, channels), strides (1, N)
    yt = torch.from_numpy(Y).to(cuda).t()
    assert not xt.is_contiguous()
    _, pc = ib.spectral(ib.OP_CSD, xt, yt, axis=0, complex_output=True, **kw)
    assert so.max_rel_err(_np(pc)[1].real, g["config_4/Pxx"]) <= 1e-5
    # reference-signature csd on the strided column view
    r = ib.csd(xt[:, 1], yt[:, 1], **kw)
    assert np.array_equal(_np(r.f), g["config_4/f"])
    assert so.max_rel_err(_np(r.Pxx), g["config_4/Pxx"]) <= 1e-5


def test_config_5_long_welch_and_segment_shards(g, cuda):
    import torch
    _, make, _, kw = CASES["config_5"]
    xh = make()
    x = torch.from_numpy(xh).to(cuda)
    r = ib.welch(x, **kw)
    assert np.array_equal(_np(r.f), g["config_5/f"])
    assert so.max_rel_err(_np(r.Pxx), g["config_5/Pxx"]) <= 1e-5
    # four segment-range shards, each given only its sample span and scaled
    # with the whole signal's segment count; their sum (what the all-reduce
    # forms) is the PSD
    W, n = 4, len(xh)
    _, S = shard.framing(n, kw["nperseg"], kw["noverlap"])
    parts = []
    for rank in range(W):
        s0, s1, lo, hi = shard.segment_shard(n, kw["nperseg"], kw["noverlap"],
                                             rank, W)
        parts.append(shard._gpu_partial(
            x[lo:hi], None, op="welch", fs=kw["fs"], window=kw["window"],
            nperseg=kw["nperseg"], noverlap=kw["noverlap"], nfft=0,
            detrend=kw["detrend"], return_onesided=True, scaling="density",
            n_seg_local=s1 - s0, n_seg_total=S))
    out = sum(parts)
    assert so.max_rel_err(_np(out), g["config_5/Pxx"]) <= 1e-5
