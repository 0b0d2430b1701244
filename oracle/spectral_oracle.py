"""CPU oracle for the spectral hot path — test infrastructure only.

A numpy restatement of the reference frontend's algorithm
(src/ops/signal/spectral_analysis.cpp), used by tests/, by
``__graft_entry__.smoke()`` and by ``bench.py``'s CPU baseline to check the
B200 kernels.  It is never imported by the product package.

Pinned by: the reference's own known-answer tests for the sub-steps
(windows vs scipy at atol 1e-10, tests/python_align/cpu/test_signal.py:50-70;
FFT vs numpy at atol 1e-8, tests/python_align/cpu/test_fft.py:26-48) and by
golden vectors produced by the reference itself, compiled here from its
sources (oracle/Makefile, tests/golden/make_golden.py).

The reference's FFT is FFTW3 (``fftw_plan_many_dft`` / ``fftw_execute_dft``,
backends/cpu/kernels/fft/fft_c2c.cpp:44-59; "FFTW 3.3+", README.md:237), an
external library absent here; its published algorithm is the unnormalised
forward DFT X[k] = sum_n x[n] exp(-2 pi i k n / N), which numpy.fft.fft
computes (in float64 here).
"""
from __future__ import annotations

import math

import numpy as np

# ---------------------------------------------------------------------------
# Windows: src/ops/signal/windows.cpp
# ---------------------------------------------------------------------------


def _apply_sym(M, sym, fn):
    # windows.cpp:25-36
    if M < 1:
        raise ValueError("window: M must be >= 1")
    if M == 1:
        return np.ones(1)
    Mw = M if sym else M + 1
    w = fn(Mw)
    return w[:M]


def _cosine_sum(N, a):
    # windows.cpp:40-55: w = a0 + sum_k (-1)^k a_k cos(n * (2 pi k / (N-1)))
    den = N - 1.0
    i = np.arange(N, dtype=np.float64)
    r = np.full(N, a[0])
    for k in range(1, len(a)):
        sign = 1.0 if k % 2 == 0 else -1.0
        c = 2.0 * math.pi * k / den
        r = r + np.cos(i * c) * (sign * a[k])
    return r


def get_window(name, M, fftbins=False):
    """get_window (windows.cpp:557-601); fftbins=False -> symmetric."""
    sym = not fftbins
    if name in ("boxcar", "rect", "ones", "dirichlet"):
        return _apply_sym(M, sym, lambda N: np.ones(N))
    if name == "hann" or name == "hanning":               # :265
        return _apply_sym(M, sym, lambda N: _cosine_sum(N, [0.5, 0.5]))
    if name == "hamming":                                   # :279-287
        def f(N):
            i = np.arange(N, dtype=np.float64)
            return 0.54 + (-0.46) * np.cos(i * (2.0 * math.pi / (N - 1)))
        return _apply_sym(M, sym, f)
    if name == "blackman":                                  # :232-234
        return _apply_sym(M, sym, lambda N: _cosine_sum(N, [0.42, 0.50, 0.08]))
    if name == "nuttall":
        return _apply_sym(M, sym, lambda N: _cosine_sum(
            N, [0.3635819, 0.4891775, 0.1365995, 0.0106411]))
    if name == "blackmanharris":
        return _apply_sym(M, sym, lambda N: _cosine_sum(
            N, [0.35875, 0.48829, 0.14128, 0.01168]))
    if name == "flattop":
        return _apply_sym(M, sym, lambda N: _cosine_sum(
            N, [0.21557895, 0.41663158, 0.277263158, 0.083578947, 0.006947368]))
    if name == "bartlett":                                  # :189-200
        def f(N):
            i = np.arange(N, dtype=np.float64)
            ramp = (i * 2.0) / (N - 1.0)
            return np.where(i <= float(N // 2), ramp, 2.0 - ramp)
        return _apply_sym(M, sym, f)
    if name == "cosine":                                    # :206-214
        return _apply_sym(M, sym, lambda N: np.sin(
            (np.arange(N, dtype=np.float64) + 0.5) * (math.pi / N)))
    if name == "triang":                                    # :107-123
        def f(N):
            v = np.empty(N)
            odd = N % 2 == 1
            for i in range(N):
                n = i + 1
                if n <= (N + 1) // 2:
                    v[i] = (2.0 * n / (N + 1.0)) if odd else ((2.0 * n - 1.0) / N)
                else:
                    v[i] = v[N - 1 - i]
            return v
        return _apply_sym(M, sym, f)
    raise ValueError(f"get_window: unknown window name '{name}'")


# ---------------------------------------------------------------------------
# Framing and the per-segment transform: spectral_analysis.cpp:70-96,104-171
# ---------------------------------------------------------------------------


def framing(n, nperseg, noverlap, for_spectrogram=False):
    """(step, n_seg): noverlap == 0 -> nperseg/2 (csd, :116-117) or
    nperseg/8 (spectrogram, :237-238); n_seg = (n - nperseg)/step + 1 (:124)."""
    if noverlap == 0:
        noverlap = nperseg // 8 if for_spectrogram else nperseg // 2
    step = nperseg - noverlap
    n_seg = (n - nperseg) // step + 1 if n >= nperseg else 0
    return step, n_seg


def _segments(x, nperseg, step, n_seg):
    idx = np.arange(n_seg)[:, None] * step + np.arange(nperseg)[None, :]
    return x[idx]


def _transform(x, win, nperseg, step, n_seg, nfft, detrend):
    """FFT_nfft(detrend(x_seg * win)) for every segment, float64."""
    seg = _segments(np.asarray(x, dtype=np.float64), nperseg, step, n_seg)
    xw = seg * win[None, :]                                    # :75-76
    if detrend == "constant":                                  # :79-82
        xw = xw - xw.mean(axis=1, keepdims=True)
    elif detrend == "linear_lsq":
        # the backend's native option (no reference counterpart: the
        # reference's 'linear' does not detrend): remove each windowed
        # segment's least-squares line, as scipy.signal.detrend(type='linear')
        xw = xw - lsq_line(xw)
    return np.fft.fft(xw, n=nfft, axis=1)                      # :90-91 (pads)


def lsq_line(z):
    """Least-squares line a + b n of each row of z (n = 0 .. M-1)."""
    M = z.shape[1]
    n = np.arange(M, dtype=np.float64)
    nb = (M - 1) / 2.0
    snn = np.sum((n - nb) ** 2)
    b = ((z * (n - nb)[None, :]).sum(axis=1) / snn if snn > 0
         else np.zeros(z.shape[0]))
    a = z.mean(axis=1) - b * nb
    return a[:, None] + b[:, None] * n[None, :]


def psd_scale(win, fs, scaling):
    # compute_psd_scale (:57-67): (fs if density else 1) / sum(w^2).
    # Note: this is the reference's formula (SciPy uses 1/(fs*sum(w^2))).
    return (fs if scaling == "density" else 1.0) / float(np.sum(win * win))


def onesided_mask(F, nfft, onesided):
    m = np.ones(F)
    if onesided and nfft > 1:                                  # :157-166
        m[1:F - 1] = 2.0
    return m


def csd_sums(x, y, nperseg, noverlap, nfft, detrend, seg_range=None, window="hann",
             win=None, onesided=True):
    """Unscaled sum over segments of conj(X_s) * Y_s (complex), and n_seg."""
    n = len(x)
    nfft = nfft or nperseg
    step, n_seg = framing(n, nperseg, noverlap)
    if win is None:
        win = get_window(window, nperseg, False)
    s0, s1 = seg_range if seg_range is not None else (0, n_seg)
    xs = np.asarray(x, dtype=np.float64)[s0 * step:]
    ys = np.asarray(y, dtype=np.float64)[s0 * step:]
    X = _transform(xs, win, nperseg, step, s1 - s0, nfft, detrend)
    Y = X if y is x else _transform(ys, win, nperseg, step, s1 - s0, nfft, detrend)
    F = nfft // 2 + 1 if onesided else nfft
    return (np.conj(X) * Y).sum(axis=0)[:F], n_seg


def csd(x, y, fs=1.0, window="hann", nperseg=256, noverlap=0, nfft=0,
        detrend="constant", return_onesided=True, scaling="density",
        complex_output=False, win=None):
    """Reference csd (:104-171). Returns (f, Pxy); Pxy is Re(.) as the
    reference returns, or the complex cross spectrum with complex_output."""
    nfft = nfft or nperseg
    step, n_seg = framing(len(x), nperseg, noverlap)
    if n_seg < 1:
        raise ValueError("csd: signal too short for given nperseg")
    if win is None:
        win = get_window(window, nperseg, False)
    F = nfft // 2 + 1 if return_onesided else nfft
    sums, _ = csd_sums(x, y, nperseg, noverlap, nfft, detrend, win=win,
                       onesided=return_onesided)
    scale = psd_scale(win, fs, scaling)
    p = sums * (scale / n_seg) * onesided_mask(F, nfft, return_onesided)
    f = np.arange(F) * (fs / nfft)                             # fft_freqs :47-55
    return f, (p if complex_output else p.real)


def welch(x, fs=1.0, window="hann", nperseg=256, noverlap=0, nfft=0,
          detrend="constant", return_onesided=True, scaling="density", win=None):
    """Reference welch (:177-183) = csd(x, x)."""
    return csd(x, x, fs, window, nperseg, noverlap, nfft, detrend,
               return_onesided, scaling, win=win)


def periodogram(x, fs=1.0, window="boxcar", nfft=0, detrend="constant",
                return_onesided=True, scaling="density"):
    """Reference periodogram (:189-193) = welch with nperseg 256, noverlap 0
    (hence the default 128)."""
    return welch(x, fs, window, 256, 0, nfft, detrend, return_onesided, scaling)


def coherence(x, y, fs=1.0, window="hann", nperseg=256, noverlap=0, nfft=0,
              detrend="constant"):
    """Reference coherence (:199-221): Pxx, Pyy from welch, Pxy the real part
    csd returns; Cxy = Pxy^2 / max(Pxx Pyy, 1e-30), 0 where Pxx Pyy <= 1e-30."""
    f, pxx = welch(x, fs, window, nperseg, noverlap, nfft, detrend)
    _, pyy = welch(y, fs, window, nperseg, noverlap, nfft, detrend)
    _, pxy = csd(x, y, fs, window, nperseg, noverlap, nfft, detrend)
    den = pxx * pyy
    eps = 1e-30
    cxy = pxy * pxy / np.maximum(den, eps)
    return f, np.where(den <= eps, 0.0, cxy)


def spectrogram(x, fs=1.0, window="hann", nperseg=256, noverlap=0, nfft=0,
                detrend="constant", return_onesided=True, mode="psd",
                complex_output=False, win=None):
    """Reference spectrogram (:227-324).  Returns (f, t, Sxx) with Sxx of
    shape (n_seg, n_freq) as the reference's transposed view; with
    complex_output the complex X of shape (n_freq, n_seg)."""
    nfft = nfft or nperseg
    step, n_seg = framing(len(x), nperseg, noverlap, for_spectrogram=True)
    if n_seg < 1:
        raise ValueError("spectrogram: signal too short")
    if win is None:
        win = get_window(window, nperseg, False)
    F = nfft // 2 + 1 if return_onesided else nfft
    X = _transform(x, win, nperseg, step, n_seg, nfft, detrend)[:, :F]
    t = (np.arange(n_seg) * step + nperseg / 2.0) / fs          # :250-253
    f = np.arange(F) * (fs / nfft)
    if complex_output:
        return f, t, X.T
    if mode == "psd":
        s = (X.real ** 2 + X.imag ** 2) * psd_scale(win, fs, "density")
        s = s * onesided_mask(F, nfft, return_onesided)[None, :]
    elif mode == "complex":
        s = X.real
    else:
        s = np.abs(X)
    return f, t, s


def stft(x, fs=1.0, window="hann", nperseg=256, noverlap=0, nfft=0,
         complex_output=False, win=None):
    """Reference stft (:330-334) = spectrogram(detrend none, onesided,
    mode complex): Re(X) (n_seg, n_freq); complex_output gives X (F, S)."""
    return spectrogram(x, fs, window, nperseg, noverlap, nfft, "none", True,
                       "complex", complex_output=complex_output, win=win)


def istft(Zxx, fs=1.0, window="hann", nperseg=0, noverlap=0, nfft=0,
          reference_mirror=False):
    """Reference istft (:340-457): per frame Re(ifft(full, nfft))[:nperseg]
    * w, where full mirrors bins 1..F-2 as conjugates when F == nfft/2 + 1
    and nfft > 2; overlap-add with hop = nperseg - noverlap; division by the
    overlap-added w^2 where it exceeds 1e-10.  fs is unused (as there).

    reference_mirror=True reproduces what the reference computes instead of
    the mirror it intends: it conjugates the view col[1:F-1] with an
    elementwise op that reads from the storage base and ignores the view's
    offset (:384-389), so full[nfft-m] = conj(Z[m-1]) rather than
    conj(Z[m]).  The backend computes the intended inverse."""
    Z = np.asarray(Zxx, dtype=np.complex128)
    F, S = Z.shape
    if nfft <= 0:
        nfft = 2 * (F - 1)
    if nperseg <= 0:
        nperseg = nfft
    if noverlap <= 0:
        noverlap = nperseg // 2
    win = get_window(window, nperseg, False)
    hop = nperseg - noverlap
    if F == nfft // 2 + 1 and nfft > 2:
        lo = 0 if reference_mirror else 1
        full = np.concatenate([Z, np.conj(Z[lo:lo + F - 2][::-1])], axis=0)
    else:
        full = Z
    seg = np.fft.ifft(full, n=nfft, axis=0).real[:nperseg] * win[:, None]
    n_total = (S - 1) * hop + nperseg
    out = np.zeros(n_total)
    norm = np.zeros(n_total)
    for i in range(S):
        out[i * hop:i * hop + nperseg] += seg[:, i]
        norm[i * hop:i * hop + nperseg] += win * win
    m = np.abs(norm) > 1e-10
    out[m] /= norm[m]
    return out


def max_rel_err(got, ref):
    """max_k |got - ref| / max_k |ref| (the parity metric)."""
    got = np.asarray(got)
    ref = np.asarray(ref)
    den = np.max(np.abs(ref))
    if den == 0:
        return float(np.max(np.abs(got)))
    return float(np.max(np.abs(got - ref)) / den)


def reference_spectrogram_layout(s, mode, nfft, onesided=True):
    """What the reference's spectrogram returns given the intended (n_seg,
    n_freq) result `s` (psd values before the one-sided mask).

    The reference writes each column with scatter(Sxx_2d, 1, col_idx, col)
    and a 1-D index (spectral_analysis.cpp:294-299); the CPU scatter kernel
    unravels the index position with the output's dims
    (backends/cpu/kernels/indexing/scatter_reduce.cpp), so for segment j only
    rows r = 0..(F-1)//S are written, with Sxx_2d[r, j] = col[min((r+1)*S, F) - 1]
    (last write wins).  The psd mask then scales row r by mask[r] (:306-315).
    With a single segment every row is written and the result is exact.
    """
    S, F = s.shape
    out = np.zeros((S, F))
    mask = onesided_mask(F, nfft, onesided) if mode == "psd" else np.ones(F)
    for r in range((F - 1) // S + 1):
        k = min((r + 1) * S, F) - 1
        out[:, r] = s[:, k] * mask[r]
    return out
