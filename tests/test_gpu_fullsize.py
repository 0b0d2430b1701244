"""Parity on the GPU against the reference's golden vectors and, at the full
benchmark sizes, against an f64 restatement of the oracle's algorithm.

* Golden: every case of tests/golden/reference_cases.npz (outputs of the
  reference itself) through the C ABI, with the parity bar of the oracle
  tests (bit-exact axes, 1e-5 / 1e-12 of the max bin).
* Full size: the five benchmark workloads at their real shapes.  The numpy
  oracle is too slow there, so its algorithm (window, detrend after the
  window, FFT, |X|^2 or conj(X)Y, segment mean, scale, one-sided mask —
  oracle.spectral_oracle._transform / csd / spectrogram) is restated with
  torch f64 ops, channel chunk by channel chunk, as a checker only.
"""
import json
import os

import numpy as np
import pytest

import insight_b200 as ib
from insight_b200 import shard
from oracle import spectral_oracle as so

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def _cases():
    with open(os.path.join(GOLDEN, "reference_cases.json")) as f:
        return json.load(f)


@pytest.fixture(scope="module")
def golden():
    return np.load(os.path.join(GOLDEN, "reference_cases.npz"))


def _np(a):
    return a.detach().cpu().numpy() if hasattr(a, "detach") else np.asarray(a)


@pytest.mark.parametrize("case", _cases(), ids=lambda c: c["name"])
def test_golden_case_on_gpu(case, golden, cuda):
    import torch
    name, op, kw = case["name"], case["op"], dict(case["kwargs"])
    x = golden[name + "/x"]
    xg = torch.from_numpy(x).to(cuda)
    tol = 1e-5 if x.dtype == np.float32 else 1e-12
    if op == "istft":
        # the reference mirrors a one-sided Zxx one bin off (its conj ignores
        # the slice offset); the backend computes the intended inverse, which
        # equals the reference wherever no mirroring happens (two-sided input)
        z = golden[name + "/Zxx"]
        ik = {k: v for k, v in kw.items() if k != "stft"}
        got = _np(ib.istft(torch.from_numpy(z).to(cuda), **ik))
        nfft = ik.get("nfft", 0) or 2 * (z.shape[0] - 1)
        if z.shape[0] == nfft // 2 + 1:
            expect = so.istft(z, **ik)
        else:
            expect = golden[name + "/out"]
        # compared before the division by the overlap-added squared window,
        # which amplifies rounding at the window's ends (ill-conditioned there)
        nps = ik.get("nperseg", 0) or nfft
        hop = nps - (ik.get("noverlap", 0) or nps // 2)
        w2 = so.get_window(ik.get("window", "hann"), nps) ** 2
        nrm = np.zeros(len(expect))
        for i in range(z.shape[1]):
            nrm[i * hop:i * hop + nps] += w2
        assert so.max_rel_err(got * nrm, expect * nrm) <= 1e-12
        return
    if op in ("welch", "csd", "coherence", "periodogram"):
        if op == "welch":
            r = ib.welch(xg, **kw)
        elif op == "periodogram":
            r = ib.periodogram(xg, **kw)
        else:
            yg = torch.from_numpy(golden[name + "/y"]).to(cuda)
            r = (ib.csd if op == "csd" else ib.coherence)(xg, yg, **kw)
        p = r.Pxx
        assert np.array_equal(_np(r.f), golden[name + "/f"])
        assert so.max_rel_err(_np(p), golden[name + "/Pxx"]) <= tol
        return
    nfft = kw.get("nfft", 0) or kw["nperseg"]
    if op == "stft":
        r = ib.stft(xg, **kw)
        mode = "complex"
    else:
        r = ib.spectrogram(xg, **kw)
        mode = kw.get("mode", "psd")
    s = _np(r.Sxx)
    if mode == "psd":
        s = s / so.onesided_mask(s.shape[1], nfft, True)[None, :]
    assert np.array_equal(_np(r.f), golden[name + "/f"])
    assert np.array_equal(_np(r.t), golden[name + "/t"])
    expect = so.reference_spectrogram_layout(s, mode, nfft)
    assert so.max_rel_err(expect, golden[name + "/Sxx"]) <= tol


# ------------------------------------------------------------ full size ----
class _Err:
    """Running max |got - ref| and max |ref| over chunks (max_rel_err)."""

    def __init__(self):
        self.num = 0.0
        self.den = 0.0

    def add(self, got, ref):
        self.num = max(self.num, float((got - ref).abs().max()))
        self.den = max(self.den, float(ref.abs().max()))

    @property
    def rel(self):
        return self.num / self.den


def _spectra(torch, xs, win, detrend):
    """rfft(detrend(x_seg * w)) of a (..., S, L) f64 block of segments."""
    z = xs * win
    if detrend == "constant":
        z = z - z.mean(dim=-1, keepdim=True)
    return torch.fft.rfft(z, dim=-1)


def test_stft_full_size(cuda):
    """signal::stft, 64 ch x 2^22 f32, nperseg 2048, hop 512, hann, complex64."""
    import torch
    C, N, L, H, fs = 64, 1 << 22, 2048, 512, 1.0e4
    g = torch.Generator(device=cuda)
    g.manual_seed(1001)
    x = torch.randn((C, N), generator=g, device=cuda, dtype=torch.float32)
    t = torch.arange(N, device=cuda, dtype=torch.float64) / fs
    x += torch.cos(2 * np.pi * (0.5 * (0.4 * fs / (N / fs)) * t * t)).float()[None]
    r = ib.stft(x, fs=fs, window="hann", nperseg=L, noverlap=L - H,
                complex_output=True)
    step, S = so.framing(N, L, L - H, for_spectrogram=True)
    F = L // 2 + 1
    assert tuple(r.Sxx.shape) == (C, F, S) and r.Sxx.dtype == torch.complex64
    assert np.array_equal(_np(r.f), np.arange(F) * (fs / L))
    assert np.array_equal(_np(r.t), (np.arange(S) * step + L / 2.0) / fs)
    win = torch.from_numpy(so.get_window("hann", L)).to(cuda)
    err = _Err()
    for c in range(C):
        ref = _spectra(torch, x[c].double().unfold(0, L, H), win, "none")
        err.add(r.Sxx[c].to(torch.complex128).t(), ref)
    assert err.rel <= 1e-5, err.rel


def test_welch_f64_full_size(cuda):
    """signal::welch f64, 1024 ch x 2^20, nperseg 4096, 50%, hamming,
    detrend 'linear' (no detrend, as the reference)."""
    import torch
    C, N, L = 1024, 1 << 20, 4096
    g = torch.Generator(device=cuda)
    g.manual_seed(1002)
    x = torch.randn((C, N), generator=g, device=cuda, dtype=torch.float64)
    # AR(1)-like colour without a long recursion: x[n] + 0.9 x[n-1]
    x[:, 1:] += 0.9 * x[:, :-1].clone()
    r = ib.welch(x, fs=1.0, window="hamming", nperseg=L, detrend="linear")
    win_np = so.get_window("hamming", L)
    win = torch.from_numpy(win_np).to(cuda)
    step, S = so.framing(N, L, 0)
    F = L // 2 + 1
    k = torch.from_numpy(so.psd_scale(win_np, 1.0, "density") / S *
                         so.onesided_mask(F, L, True)).to(cuda)
    err = _Err()
    for c0 in range(0, C, 16):
        X = _spectra(torch, x[c0:c0 + 16].unfold(1, L, step), win, "none")
        ref = (X.real ** 2 + X.imag ** 2).sum(dim=1) * k
        err.add(r.Pxx[c0:c0 + 16], ref)
    assert err.rel <= 1e-12, err.rel


def test_csd_full_size_transposed(cuda):
    """signal::csd, 512 f32 pairs x 2^21 as (N, C) transposed views,
    nperseg 2048, 50%, hann, complex64 cross spectra."""
    import torch
    C, N, L = 512, 1 << 21, 2048
    g = torch.Generator(device=cuda)
    g.manual_seed(1003)
    x = torch.randn((C, N), generator=g, device=cuda, dtype=torch.float32)
    y = 0.7 * torch.roll(x, 17, dims=1) + 0.3 * torch.randn(
        (C, N), generator=g, device=cuda, dtype=torch.float32)
    xt, yt = x.t(), y.t()
    f, p = ib.spectral(ib.OP_CSD, xt, yt, fs=1.0, window="hann", nperseg=L,
                       axis=0, complex_output=True)
    F = L // 2 + 1
    assert tuple(p.shape) == (C, F) and p.dtype == torch.complex64
    win_np = so.get_window("hann", L)
    win = torch.from_numpy(win_np).to(cuda)
    step, S = so.framing(N, L, 0)
    k = torch.from_numpy(so.psd_scale(win_np, 1.0, "density") / S *
                         so.onesided_mask(F, L, True)).to(cuda)
    err = _Err()
    for c0 in range(0, C, 8):
        X = _spectra(torch, x[c0:c0 + 8].double().unfold(1, L, step), win,
                     "constant")
        Y = _spectra(torch, y[c0:c0 + 8].double().unfold(1, L, step), win,
                     "constant")
        ref = (X.conj() * Y).sum(dim=1) * k
        err.add(p[c0:c0 + 8].to(torch.complex128), ref)
    assert err.rel <= 1e-5, err.rel


def test_istft_round_trip_full_size(cuda):
    """signal::stft of the 64 ch x 2^22 f32 workload (complex64), then istft
    with the same window and hop: the reference's normalised overlap-add
    returns the signal wherever the summed squared window exceeds 1e-10."""
    import torch
    C, N, L, H = 64, 1 << 22, 2048, 512
    g = torch.Generator(device=cuda)
    g.manual_seed(1006)
    x = torch.randn((C, N), generator=g, device=cuda, dtype=torch.float32)
    z = ib.stft(x, window="hann", nperseg=L, noverlap=L - H,
                complex_output=True).Sxx
    y = ib.istft(z, window="hann", nperseg=L, noverlap=L - H)
    S = z.shape[-1]
    n_total = (S - 1) * H + L
    assert tuple(y.shape) == (C, n_total) and y.dtype == torch.float64
    # interior samples (the symmetric hann window is 0 at the segment ends)
    err = (y[:, H:n_total - H] - x[:, H:n_total - H].double()).abs().max()
    assert float(err) <= 1e-5 * float(x.abs().max()), float(err)
    del z, y


def test_welch_long_full_size_and_segment_shards(cuda):
    """signal::welch of one f32 signal of 2^30 samples, nperseg 8192,
    noverlap 4096, blackman: the one-call result, the result of 8
    segment-range shards (each given only its sample span, partial sums
    reduced on the host as the all-reduce would), and the f64 restatement."""
    import torch
    N, L, H = 1 << 30, 8192, 4096
    g = torch.Generator(device=cuda)
    g.manual_seed(1005)
    x = torch.randn(N, generator=g, device=cuda, dtype=torch.float32)
    kw = dict(fs=1.0, window="blackman", nperseg=L, noverlap=L - H,
              detrend="constant")
    one = ib.welch(x, **kw).Pxx

    W = 8
    _, S_all = shard.framing(N, L, L - H)
    parts = []
    for rk in range(W):
        s0, s1, lo, hi = shard.segment_shard(N, L, L - H, rk, W)
        parts.append(shard._gpu_partial(x[lo:hi], None, op="welch", nfft=0,
                                        return_onesided=True, scaling="density",
                                        n_seg_local=s1 - s0, n_seg_total=S_all,
                                        **kw))
    total = torch.stack(parts).sum(dim=0)

    def _sum_all(t):
        t.copy_(total)

    _, _, lo0, hi0 = shard.segment_shard(N, L, L - H, 0, W)
    sharded = shard.welch_segment_sharded(x[lo0:hi0], N, rank=0, world=W,
                                          all_reduce=_sum_all, **kw)
    # both sum f32 transforms in f64; only the unit boundaries differ
    assert so.max_rel_err(_np(sharded), _np(one)) <= 1e-6

    win_np = so.get_window("blackman", L)
    win = torch.from_numpy(win_np).to(cuda)
    step, S = so.framing(N, L, L - H)
    F = L // 2 + 1
    segs = x.unfold(0, L, step)
    acc = torch.zeros(F, device=cuda, dtype=torch.float64)
    for s0 in range(0, S, 8192):
        X = _spectra(torch, segs[s0:s0 + 8192].double(), win, "constant")
        acc += (X.real ** 2 + X.imag ** 2).sum(dim=0)
    ref = acc * torch.from_numpy(so.psd_scale(win_np, 1.0, "density") / S *
                                 so.onesided_mask(F, L, True)).to(cuda)
    assert so.max_rel_err(_np(one), _np(ref)) <= 1e-5
