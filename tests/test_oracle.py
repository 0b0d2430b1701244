"""Pins the CPU oracle before it is trusted (no GPU needed).

1. Known-answer tests the reference holds for the sub-steps:
   symmetric windows vs scipy.signal.windows at atol 1e-10
   (reference tests/python_align/cpu/test_signal.py:50-70) and the FFT vs
   numpy at atol 1e-8 (tests/python_align/cpu/test_fft.py:26-48; here vs the
   DFT definition).
2. Golden vectors produced by the reference itself (tests/golden/, made by
   tests/golden/make_golden.py from the reference compiled from its sources).
3. When oracle/_ref is built, fresh random cases against the live reference.
"""
import json
import os

import numpy as np
import pytest

from oracle import ref_runner
from oracle import spectral_oracle as so

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


@pytest.mark.parametrize("name", ["hann", "hamming", "blackman", "boxcar",
                                  "bartlett", "nuttall", "blackmanharris",
                                  "flattop", "cosine", "triang"])
@pytest.mark.parametrize("M", [1, 7, 64, 255, 1024])
def test_windows_vs_scipy(name, M):
    sw = pytest.importorskip("scipy.signal.windows")
    if name == "bartlett" and M % 2 == 0:
        # the reference's bartlett keeps the rising ramp through i == N/2
        # (windows.cpp:189-200), which differs from scipy for even M
        pytest.skip("reference bartlett differs from scipy for even M")
    ref = sw.get_window(name, M, fftbins=False)
    assert np.allclose(so.get_window(name, M), ref, atol=1e-10, rtol=0)


@pytest.mark.parametrize("n", [8, 16, 60, 128])
def test_transform_is_the_dft(n):
    rng = np.random.default_rng(n)
    x = rng.standard_normal(n)
    win = np.ones(n)
    X = so._transform(x, win, n, n, 1, n, "none")[0]
    k = np.arange(n)
    D = np.exp(-2j * np.pi * np.outer(k, k) / n)
    assert np.allclose(X, D @ x, atol=1e-8)


@pytest.mark.parametrize("M", [2, 7, 256, 1000])
def test_lsq_detrend_matches_scipy(M):
    """The native 'linear_lsq' option has no reference counterpart; its
    restatement is pinned to scipy.signal.detrend(type='linear')."""
    sig = pytest.importorskip("scipy.signal")
    rng = np.random.default_rng(M)
    z = rng.standard_normal((5, M)) + 3.0 + 0.01 * np.arange(M)[None, :]
    got = z - so.lsq_line(z)
    ref = sig.detrend(z, axis=1, type="linear")
    assert np.allclose(got, ref, atol=1e-12, rtol=0)


def _cases():
    with open(os.path.join(GOLDEN, "reference_cases.json")) as f:
        return json.load(f)


@pytest.fixture(scope="module")
def golden():
    return np.load(os.path.join(GOLDEN, "reference_cases.npz"))


@pytest.mark.parametrize("case", _cases(), ids=lambda c: c["name"])
def test_oracle_matches_reference_golden(case, golden):
    name, op, kw = case["name"], case["op"], dict(case["kwargs"])
    x = golden[name + "/x"]
    if op == "istft":
        ik = {k: v for k, v in kw.items() if k != "stft"}
        got = so.istft(golden[name + "/Zxx"], reference_mirror=True, **ik)
        assert so.max_rel_err(got, golden[name + "/out"]) <= 1e-12
        return
    if op in ("welch", "csd", "coherence", "periodogram"):
        if op == "welch":
            f, p = so.welch(x, **kw)
        elif op == "periodogram":
            f, p = so.periodogram(x, **kw)
        elif op == "coherence":
            f, p = so.coherence(x, golden[name + "/y"], **kw)
        else:
            f, p = so.csd(x, golden[name + "/y"], **kw)
        assert np.array_equal(f, golden[name + "/f"])
        assert so.max_rel_err(p, golden[name + "/Pxx"]) <= 1e-12
        return
    mode = kw.get("mode", "psd") if op == "spectrogram" else "complex"
    if op == "stft":
        f, t, s = so.stft(x, **kw)
        nfft = kw.get("nfft", 0) or kw["nperseg"]
    else:
        f, t, s = so.spectrogram(x, **kw)
        nfft = kw.get("nfft", 0) or kw["nperseg"]
    if mode == "psd":
        s = s / so.onesided_mask(s.shape[1], nfft, True)[None, :]
    expect = so.reference_spectrogram_layout(s, mode, nfft)
    assert np.array_equal(f, golden[name + "/f"])
    assert np.array_equal(t, golden[name + "/t"])
    tol = 1e-5 if x.dtype == np.float32 else 1e-12
    assert so.max_rel_err(expect, golden[name + "/Sxx"]) <= tol
    if s.shape[0] == 1:
        # single segment: the reference writes the whole column
        full = s * (so.onesided_mask(s.shape[1], nfft, True)[None, :]
                    if mode == "psd" else 1.0)
        assert so.max_rel_err(full, golden[name + "/Sxx"]) <= tol


needs_ref = pytest.mark.skipif(not ref_runner.available(),
                               reason="oracle/_ref not built")


@needs_ref
@pytest.mark.parametrize("seed", range(6))
def test_oracle_vs_live_reference(seed):
    rng = np.random.default_rng(seed)
    L = int(rng.choice([16, 32, 64, 128, 256]))
    n = int(rng.integers(L, 12 * L))
    window = str(rng.choice(["hann", "hamming", "blackman"]))
    detrend = str(rng.choice(["constant", "none", "linear"]))
    nfft = int(rng.choice([0, 2 * L]))
    x = rng.standard_normal(n)
    y = rng.standard_normal(n)
    kw = dict(fs=float(rng.uniform(0.5, 100)), window=window, nperseg=L, nfft=nfft,
              detrend=detrend)
    f, p = ref_runner.welch(x, **kw)
    f2, p2 = so.welch(x, **kw)
    assert np.array_equal(f, f2) and so.max_rel_err(p2, p) <= 1e-12
    f, p = ref_runner.csd(x, y, **kw)
    f2, p2 = so.csd(x, y, **kw)
    assert so.max_rel_err(p2, p) <= 1e-12
    # single-segment spectrogram: every bin is written by the reference
    xs = x[:L]
    f, t, s = ref_runner.spectrogram(xs, window=window, nperseg=L, nfft=nfft,
                                     mode="complex", detrend=detrend)
    f2, t2, s2 = so.spectrogram(xs, window=window, nperseg=L, nfft=nfft,
                                mode="complex", detrend=detrend)
    assert so.max_rel_err(s2, s) <= 1e-12


def test_reference_f32_welch_throws_as_documented():
    if not ref_runner.available():
        pytest.skip("oracle/_ref not built")
    with pytest.raises(RuntimeError, match="item<float64>"):
        ref_runner.welch(np.zeros(1024, np.float32), nperseg=256)


# ------------------------------------------- configuration-scale fixtures --
import sys as _sys  # noqa: E402

_sys.path.insert(0, GOLDEN)
import config_inputs as _ci  # noqa: E402


@pytest.fixture(scope="module")
def config_golden():
    return np.load(os.path.join(GOLDEN, "reference_configs.npz"))


@pytest.mark.parametrize("case", _ci.CASES, ids=lambda c: c[0])
def test_oracle_matches_reference_at_config_parameters(case, config_golden):
    """The restatement against the reference's own outputs at the benchmark
    configurations' nperseg, windows, overlaps and detrend (one channel or
    pair each, inputs promoted to F64 as the reference needs)."""
    name, make, op, kw = case
    g = config_golden
    if op == "csd":
        x, y = make()
        f, p = so.csd(x.astype(np.float64), y.astype(np.float64), **kw)
    elif op == "welch":
        f, p = so.welch(make().astype(np.float64), **kw)
    else:
        f, t, s = so.stft(make().astype(np.float64), **kw)
        assert np.array_equal(t, g[name + "/t"])
        expect = so.reference_spectrogram_layout(s, "complex", kw["nperseg"])
        assert np.array_equal(f, g[name + "/f"])
        assert so.max_rel_err(expect, g[name + "/Sxx"]) <= 1e-12
        return
    assert np.array_equal(f, g[name + "/f"])
    assert so.max_rel_err(p, g[name + "/Pxx"]) <= 1e-12
