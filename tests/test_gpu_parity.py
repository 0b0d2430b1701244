"""Parity of the fused sm_100a kernels with the CPU oracle, through the C ABI.

Every call goes through libinsight_b200_backend.so (insight_b200.signal is a
ctypes mirror of the reference's Python API).  Tolerances are the parity bar:
max_k |P - P_ref| / max_k |P_ref| <= 1e-5 for f32 and <= 1e-12 for f64;
frequency and time axes and segment counts must be bit-exact.
"""
import numpy as np
import pytest

import insight_b200 as ib
from oracle import spectral_oracle as so

pytestmark = pytest.mark.gpu

TOL = {np.float32: 1e-5, np.float64: 1e-12}


def _sig(n, dtype, seed):
    rng = np.random.default_rng(seed)
    t = np.arange(n)
    x = rng.standard_normal(n) + np.sin(2 * np.pi * 0.05 * t) + 0.5 * np.sin(
        2 * np.pi * 0.31 * t)
    return x.astype(dtype)


def _np(a):
    return a.detach().cpu().numpy() if hasattr(a, "detach") else np.asarray(a)


def _to_gpu(x, cuda):
    import torch
    return torch.from_numpy(np.ascontiguousarray(x)).to(cuda)


# ---------------------------------------------------------------- welch ----
@pytest.mark.parametrize("dtype", [np.float32, np.float64])
@pytest.mark.parametrize("nperseg,nfft,window,detrend", [
    (16, 0, "hann", "constant"),
    (64, 0, "hamming", "constant"),
    (256, 0, "hann", "constant"),
    (1024, 0, "hann", "constant"),
    (2048, 0, "blackman", "none"),
    (4096, 0, "hamming", "linear"),
    (8192, 0, "blackman", "constant"),
    (100, 128, "hann", "constant"),     # zero padded, frequency-domain detrend
    (200, 512, "hamming", "none"),
])
def test_welch(cuda, dtype, nperseg, nfft, window, detrend):
    n = max(6 * nperseg + 37, 3000)
    x = _sig(n, dtype, nperseg)
    r = ib.welch(_to_gpu(x, cuda), fs=1e4, window=window, nperseg=nperseg,
                 nfft=nfft, detrend=detrend)
    f, p = so.welch(x, fs=1e4, window=window, nperseg=nperseg, nfft=nfft,
                    detrend=detrend)
    assert np.array_equal(_np(r.f), f)
    assert so.max_rel_err(_np(r.Pxx), p) <= TOL[dtype]


@pytest.mark.parametrize("dtype", [np.float32, np.float64])
@pytest.mark.parametrize("onesided,scaling,noverlap", [
    (False, "density", 0), (True, "spectrum", 0), (True, "density", 200),
    (False, "spectrum", 255)])
def test_welch_options(cuda, dtype, onesided, scaling, noverlap):
    x = _sig(5001, dtype, 7)
    r = ib.welch(_to_gpu(x, cuda), fs=3.0, nperseg=256, noverlap=noverlap,
                 return_onesided=onesided, scaling=scaling)
    f, p = so.welch(x, fs=3.0, nperseg=256, noverlap=noverlap,
                    return_onesided=onesided, scaling=scaling)
    assert np.array_equal(_np(r.f), f)
    assert so.max_rel_err(_np(r.Pxx), p) <= TOL[dtype]


@pytest.mark.parametrize("dtype", [np.float32, np.float64])
def test_welch_host_arrays(dtype):
    # numpy in, numpy out: the backend copies to and from the GPU itself.
    x = _sig(1 << 16, dtype, 3)
    r = ib.welch(x, fs=1e4, nperseg=1024, noverlap=512)
    f, p = so.welch(x, fs=1e4, nperseg=1024, noverlap=512)
    assert isinstance(r.Pxx, np.ndarray)
    assert so.max_rel_err(r.Pxx, p) <= TOL[dtype]


@pytest.mark.parametrize("segments", [1, 2, 3, 17])
def test_welch_segment_counts(cuda, segments):
    # odd counts leave the last transform with a single segment
    L = 256
    n = (segments - 1) * 128 + L + 5
    x = _sig(n, np.float64, segments)
    r = ib.welch(_to_gpu(x, cuda), nperseg=L)
    f, p = so.welch(x, nperseg=L)
    assert so.max_rel_err(_np(r.Pxx), p) <= 1e-12


# ------------------------------------------------------------------ csd ----
@pytest.mark.parametrize("dtype", [np.float32, np.float64])
@pytest.mark.parametrize("nperseg,nfft,detrend,onesided", [
    (64, 0, "constant", True), (2048, 0, "constant", True),
    (512, 0, "none", False), (300, 1024, "constant", True)])
def test_csd(cuda, dtype, nperseg, nfft, detrend, onesided):
    n = 9 * nperseg + 11
    x = _sig(n, dtype, 1)
    y = (0.7 * np.roll(x.astype(np.float64), 17) + 0.3 * _sig(n, np.float64, 2)
         ).astype(dtype)
    r = ib.csd(_to_gpu(x, cuda), _to_gpu(y, cuda), fs=2.0, nperseg=nperseg,
               nfft=nfft, detrend=detrend, return_onesided=onesided)
    f, p = so.csd(x, y, fs=2.0, nperseg=nperseg, nfft=nfft, detrend=detrend,
                  return_onesided=onesided)
    assert np.array_equal(_np(r.f), f)
    assert so.max_rel_err(_np(r.Pxx), p) <= TOL[dtype]
    # complex cross spectrum (native output)
    f2, pc = ib.spectral(ib.OP_CSD, _to_gpu(x, cuda), _to_gpu(y, cuda), fs=2.0,
                         nperseg=nperseg, nfft=nfft, detrend=detrend,
                         return_onesided=onesided, complex_output=True)
    _, pr = so.csd(x, y, fs=2.0, nperseg=nperseg, nfft=nfft, detrend=detrend,
                   return_onesided=onesided, complex_output=True)
    assert so.max_rel_err(_np(pc), pr) <= TOL[dtype]


@pytest.mark.parametrize("dtype", [np.float32, np.float64])
@pytest.mark.parametrize("gain", [1e-3, 0.0])
@pytest.mark.parametrize("nperseg,nfft", [(1024, 0), (300, 512)])
def test_csd_and_coherence_with_a_quiet_or_silent_y(cuda, dtype, gain, nperseg,
                                                    nfft):
    """Each spectrum is unpacked from transforms of its own signal, so a y far
    below x (or all zeros) is exact to rounding relative to y itself."""
    n = 11 * nperseg + 5
    x = _sig(n, dtype, 7)
    y = (gain * (0.7 * np.roll(x.astype(np.float64), 3)
                 + 0.3 * _sig(n, np.float64, 8))).astype(dtype)
    kw = dict(nperseg=nperseg, nfft=nfft)
    xg, yg = _to_gpu(x, cuda), _to_gpu(y, cuda)
    _, pc = ib.spectral(ib.OP_CSD, xg, yg, complex_output=True, **kw)
    _, pr = so.csd(x, y, complex_output=True, **kw)
    if gain == 0.0:
        assert np.array_equal(_np(pc), np.zeros_like(_np(pc)))
    else:
        assert so.max_rel_err(_np(pc), pr) <= TOL[dtype]
    r = ib.coherence(xg, yg, **kw)
    _, c = so.coherence(x, y, **kw)
    if gain == 0.0:
        assert np.array_equal(_np(r.Pxx), np.zeros_like(c))
    else:
        assert so.max_rel_err(_np(r.Pxx), c) <= TOL[dtype]


@pytest.mark.parametrize("dtype", [np.float32, np.float64])
@pytest.mark.parametrize("op,nperseg,nfft", [
    ("welch", 256, 0), ("welch", 200, 512), ("welch", 4096, 0), ("welch", 16, 0),
    ("csd", 1024, 0), ("coherence", 512, 0), ("stft", 2048, 0),
    ("spectrogram", 300, 1024)])
def test_linear_lsq_detrend(cuda, dtype, op, nperseg, nfft):
    """Native 'linear_lsq' detrend (no reference counterpart) against the
    oracle's least-squares restatement (pinned to scipy)."""
    n = 7 * nperseg + 31
    t = np.arange(n)
    x = (_sig(n, np.float64, 11) + 0.002 * t - 3.0).astype(dtype)
    y = (0.5 * np.roll(x.astype(np.float64), 4) + _sig(n, np.float64, 12)
         - 0.001 * t).astype(dtype)
    kw = dict(nperseg=nperseg, nfft=nfft, detrend="linear_lsq")
    xg, yg = _to_gpu(x, cuda), _to_gpu(y, cuda)
    if op == "welch":
        _, got = ib.spectral(ib.OP_WELCH, xg, **kw)
        _, ref = so.welch(x, **kw)
    elif op == "csd":
        _, got = ib.spectral(ib.OP_CSD, xg, yg, complex_output=True, **kw)
        _, ref = so.csd(x, y, complex_output=True, **kw)
    elif op == "coherence":
        _, got = ib.spectral(ib.OP_COHERENCE, xg, yg, **kw)
        _, ref = so.coherence(x, y, **kw)
    elif op == "stft":
        _, _, got = ib.spectral(ib.OP_SPECTROGRAM, xg, mode="complex",
                                complex_output=True, **kw)
        _, _, ref = so.spectrogram(x, mode="complex", complex_output=True, **kw)
    else:
        _, _, got = ib.spectral(ib.OP_SPECTROGRAM, xg, mode="psd", **kw)
        _, _, ref = so.spectrogram(x, mode="psd", **kw)
    assert so.max_rel_err(_np(got), ref) <= TOL[dtype]
    # and it differs from no detrend (the trend is not negligible)
    if op == "welch":
        _, plain = so.welch(x, nperseg=nperseg, nfft=nfft, detrend="none")
        assert so.max_rel_err(_np(got), plain) > 1e-3


# ------------------------------------------------- coherence/periodogram ----
@pytest.mark.parametrize("dtype", [np.float32, np.float64])
@pytest.mark.parametrize("nperseg,nfft,window,detrend", [
    (64, 0, "hann", "constant"), (512, 0, "hamming", "none"),
    (2048, 0, "hann", "constant"), (8192, 0, "blackman", "constant"),
    (300, 1024, "hann", "constant"), (200, 256, "hamming", "none")])
def test_coherence(cuda, dtype, nperseg, nfft, window, detrend):
    """Fast path (nfft == nperseg) and generic path (zero padding)."""
    n = 9 * nperseg + 23
    x = _sig(n, dtype, 3)
    y = (0.6 * np.roll(x.astype(np.float64), 9) + 0.4 * _sig(n, np.float64, 4)
         ).astype(dtype)
    kw = dict(fs=3.0, window=window, nperseg=nperseg, nfft=nfft, detrend=detrend)
    r = ib.coherence(_to_gpu(x, cuda), _to_gpu(y, cuda), **kw)
    f, c = so.coherence(x, y, **kw)
    assert np.array_equal(_np(r.f), f)
    assert so.max_rel_err(_np(r.Pxx), c) <= TOL[dtype]
    assert np.all(_np(r.Pxx) >= 0) and np.all(_np(r.Pxx) <= 1 + 1e-6)


@pytest.mark.parametrize("layout", ["transposed_view", "interleaved", "host"])
def test_coherence_batched(cuda, layout):
    import torch
    C, N, L = 5, 30000, 1024
    rng = np.random.default_rng(21)
    X = rng.standard_normal((C, N)).astype(np.float32)
    Y = (0.5 * np.roll(X, 3, axis=1) + 0.5 * rng.standard_normal((C, N))
         ).astype(np.float32)
    if layout == "transposed_view":   # (N, C) views, unit sample stride
        xt, yt = _to_gpu(X, cuda).t(), _to_gpu(Y, cuda).t()
    elif layout == "interleaved":     # (N, C) contiguous: sample stride C
        xt, yt = _to_gpu(X.T.copy(), cuda), _to_gpu(Y.T.copy(), cuda)
    else:                             # host arrays, (C, N)
        xt, yt = X.T.copy(), Y.T.copy()
    f, c = ib.spectral(ib.OP_COHERENCE, xt, yt, nperseg=L, axis=0)
    c = _np(c)
    assert c.shape == (C, L // 2 + 1)
    for ch in range(C):
        _, cr = so.coherence(X[ch], Y[ch], nperseg=L)
        assert so.max_rel_err(c[ch], cr) <= 1e-5
    if layout != "host":
        torch.cuda.synchronize()


def test_coherence_of_identical_and_zero_signals(cuda):
    x = _sig(20000, np.float64, 5)
    r = ib.coherence(_to_gpu(x, cuda), _to_gpu(x, cuda), nperseg=256)
    c = _np(r.Pxx)
    assert c[0] == 0.0            # constant detrend empties the DC bin
    assert np.allclose(c[1:], 1.0, atol=1e-12)
    z = np.zeros_like(x)
    r = ib.coherence(_to_gpu(x, cuda), _to_gpu(z, cuda), nperseg=256)
    assert np.array_equal(_np(r.Pxx), np.zeros(129))   # Pxx Pyy <= 1e-30 -> 0


@pytest.mark.parametrize("dtype", [np.float32, np.float64])
@pytest.mark.parametrize("window,nfft,scaling,onesided", [
    ("boxcar", 0, "density", True), ("hann", 512, "spectrum", True),
    ("hamming", 0, "density", False)])
def test_periodogram(cuda, dtype, window, nfft, scaling, onesided):
    x = _sig(5000, dtype, 6)
    kw = dict(fs=7.0, window=window, nfft=nfft, scaling=scaling,
              return_onesided=onesided)
    r = ib.periodogram(_to_gpu(x, cuda), **kw)
    f, p = so.periodogram(x, **kw)
    assert np.array_equal(_np(r.f), f)
    assert so.max_rel_err(_np(r.Pxx), p) <= TOL[dtype]


# ------------------------------------------------------------------ istft ----
def _ola_norm(n_total, S, nperseg, hop, window):
    w2 = so.get_window(window, nperseg) ** 2
    nrm = np.zeros(n_total)
    for i in range(S):
        nrm[i * hop:i * hop + nperseg] += w2
    return nrm


def _istft_err(got, ref, S, nperseg, hop, window):
    """max_rel_err of the overlap-added frames before the division by the
    summed squared window: where that sum is tiny (the window's ends) the
    division amplifies any transform's rounding, in the reference as well."""
    nrm = _ola_norm(len(ref), S, nperseg, hop, window)
    return so.max_rel_err(np.asarray(got) * nrm, np.asarray(ref) * nrm)


@pytest.mark.parametrize("cdtype", [np.complex64, np.complex128])
@pytest.mark.parametrize("L,stft_ov,nperseg,noverlap,nfft,window", [
    (128, 64, 0, 0, 0, "hann"),            # reference defaults
    (2048, 1536, 2048, 1536, 0, "hann"),
    (256, 192, 256, 192, 0, "hamming"),
    (100, 50, 100, 50, 128, "hann"),       # nperseg < nfft (truncation)
    (16, 8, 16, 8, 0, "blackman"),
    (8192, 4096, 8192, 4096, 0, "hann")])
def test_istft(cuda, cdtype, L, stft_ov, nperseg, noverlap, nfft, window):
    import torch
    x = _sig(6 * max(L, 128) + 77, np.float64, 13)
    _, _, z = so.stft(x, window=window, nperseg=L, noverlap=stft_ov,
                      nfft=nfft or L, complex_output=True)
    z = z.astype(cdtype)
    kw = dict(window=window, nperseg=nperseg, noverlap=noverlap, nfft=nfft)
    got = _np(ib.istft(torch.from_numpy(np.ascontiguousarray(z)).to(cuda), **kw))
    ref = so.istft(z, **kw)
    assert got.shape == ref.shape
    nps = nperseg or 2 * (z.shape[0] - 1)
    hop = nps - (noverlap or nps // 2)
    err = _istft_err(got, ref, z.shape[1], nps, hop, window)
    assert err <= (1e-5 if cdtype == np.complex64 else 1e-12), err


@pytest.mark.parametrize("cdtype", [np.complex64, np.complex128])
@pytest.mark.parametrize("L,hop,S", [(2048, 512, 1501), (2048, 512, 1000),
                                     (1024, 256, 777), (512, 128, 2048)])
def test_istft_many_frames(cuda, cdtype, L, hop, S):
    """Hundreds of frame pairs per CTA, odd and even frame counts: the
    pipelined frame kernel's tile sequence, its last partial tile and the
    overlap-add's interior and clipped edges."""
    import torch
    x = _sig((S - 1) * hop + L, np.float64, 31)
    _, _, z = so.stft(x, nperseg=L, noverlap=L - hop, complex_output=True)
    z = z.astype(cdtype)
    assert z.shape[1] == S
    got = _np(ib.istft(torch.from_numpy(np.ascontiguousarray(z)).to(cuda),
                       nperseg=L, noverlap=L - hop))
    ref = so.istft(z, nperseg=L, noverlap=L - hop)
    assert got.shape == ref.shape
    err = _istft_err(got, ref, S, L, hop, "hann")
    assert err <= (1e-5 if cdtype == np.complex64 else 1e-12), err


@pytest.mark.parametrize("layout", ["batch", "strided_view", "host", "two_sided"])
def test_istft_layouts(cuda, layout):
    import torch
    C, L, ov = 3, 512, 384
    X = np.stack([_sig(9000, np.float64, 20 + c) for c in range(C)])
    zs = [so.stft(X[c], nperseg=L, noverlap=ov, complex_output=True)[2]
          for c in range(C)]
    Z = np.stack(zs)                                  # (C, F, S) complex128
    kw = dict(nperseg=L, noverlap=ov)
    if layout == "two_sided":
        step, S = so.framing(9000, L, ov, True)
        segs = so._segments(X[0], L, step, S) * so.get_window("hann", L)[None, :]
        zf = np.fft.fft(segs, axis=1).T               # (L, S): no mirroring
        got = _np(ib.istft(torch.from_numpy(np.ascontiguousarray(zf)).to(cuda),
                           nfft=L, **kw))
        ref = so.istft(zf, nfft=L, **kw)
        assert _istft_err(got, ref, zf.shape[1], L, L - ov, "hann") <= 1e-12
        return
    if layout == "batch":
        zin = torch.from_numpy(Z).to(cuda)
    elif layout == "strided_view":                    # (C, F, S) view of (C, S, F)
        zin = torch.from_numpy(np.ascontiguousarray(Z.transpose(0, 2, 1))).to(
            cuda).transpose(1, 2)
    else:
        zin = Z
    got = _np(ib.istft(zin, **kw))
    assert got.shape[0] == C
    for c in range(C):
        ref = so.istft(Z[c], **kw)
        assert _istft_err(got[c], ref, Z.shape[2], L, L - ov, "hann") <= 1e-12


def test_istft_reference_signature_entry(cuda):
    """insight_b200_istft (the reference's argument list) by window name."""
    import ctypes
    import torch
    from insight_b200 import _abi
    x = _sig(5000, np.float64, 30)
    _, _, z = so.stft(x, window="hamming", nperseg=256, noverlap=128,
                      complex_output=True)
    zt = torch.from_numpy(np.ascontiguousarray(z)).to(cuda)
    n_total = (z.shape[1] - 1) * 128 + 256
    out = torch.empty(n_total, dtype=torch.float64, device=cuda)
    rc = _abi.lib().insight_b200_istft(
        ctypes.byref(_abi.as_array(zt)), 1.0, b"hamming", 256, 128, 0,
        ctypes.byref(_abi.as_array(out)))
    assert rc == 0, _abi.last_error()
    ref = so.istft(z, window="hamming", nperseg=256, noverlap=128)
    assert _istft_err(_np(out), ref, z.shape[1], 256, 128, "hamming") <= 1e-12


def test_istft_errors(cuda):
    import torch
    z = torch.zeros((65, 10), dtype=torch.complex128, device=cuda)
    with pytest.raises(RuntimeError, match="noverlap must be less than nperseg"):
        ib.istft(z, nperseg=64, noverlap=64)
    with pytest.raises(RuntimeError, match="nperseg must be <= nfft"):
        ib.istft(z, nperseg=256)
    with pytest.raises(RuntimeError, match="must be complex"):
        ib.istft(torch.zeros((65, 10), dtype=torch.float64, device=cuda))


# ------------------------------------------------------ spectrogram/stft ----
@pytest.mark.parametrize("dtype", [np.float32, np.float64])
@pytest.mark.parametrize("mode", ["psd", "complex", "magnitude"])
@pytest.mark.parametrize("nperseg,nfft,detrend", [
    (128, 0, "constant"), (2048, 0, "none"), (96, 256, "constant")])
def test_spectrogram(cuda, dtype, mode, nperseg, nfft, detrend):
    n = 11 * nperseg + 3
    x = _sig(n, dtype, 5)
    r = ib.spectrogram(_to_gpu(x, cuda), fs=8.0, nperseg=nperseg, nfft=nfft,
                       detrend=detrend, mode=mode)
    f, t, s = so.spectrogram(x, fs=8.0, nperseg=nperseg, nfft=nfft,
                             detrend=detrend, mode=mode)
    assert np.array_equal(_np(r.f), f) and np.array_equal(_np(r.t), t)
    assert _np(r.Sxx).shape == s.shape
    assert so.max_rel_err(_np(r.Sxx), s) <= TOL[dtype]


@pytest.mark.parametrize("dtype", [np.float32, np.float64])
@pytest.mark.parametrize("nperseg,noverlap", [(2048, 1536), (512, 0), (1024, 1000),
                                              (1024, 512), (8192, 6144), (64, 48)])
def test_stft(cuda, dtype, nperseg, noverlap):
    x = _sig(40 * nperseg + 1, dtype, 9)
    r = ib.stft(_to_gpu(x, cuda), fs=1e3, nperseg=nperseg, noverlap=noverlap)
    f, t, s = so.stft(x, fs=1e3, nperseg=nperseg, noverlap=noverlap)
    assert np.array_equal(_np(r.t), t)
    assert so.max_rel_err(_np(r.Sxx), s) <= TOL[dtype]
    rc = ib.stft(_to_gpu(x, cuda), fs=1e3, nperseg=nperseg, noverlap=noverlap,
                 complex_output=True)
    _, _, z = so.stft(x, fs=1e3, nperseg=nperseg, noverlap=noverlap,
                      complex_output=True)
    got = _np(rc.Sxx)
    assert got.dtype == (np.complex64 if dtype == np.float32 else np.complex128)
    assert so.max_rel_err(got, z) <= TOL[dtype]


@pytest.mark.parametrize("dtype", [np.float32, np.float64])
@pytest.mark.parametrize("L", [1024, 2048, 4096])
@pytest.mark.parametrize("segments", [1, 2, 3, 9, 17, 64])
def test_stft_complex_segment_counts(cuda, dtype, L, segments):
    """The warp-specialised stft kernel at tile and unit edges: segment
    counts that leave idle transform groups, a single segment, odd counts,
    and a batch whose channels start at different sector phases."""
    import torch
    C, H = 5, L // 4
    N = L + (segments - 1) * H + (segments % 3)   # a few samples to spare
    X = np.stack([_sig(N, dtype, 40 + c) for c in range(C)])
    f, t, z = ib.spectral(ib.OP_STFT, _to_gpu(X, cuda), nperseg=L,
                          noverlap=L - H, complex_output=True)
    z = _np(z)
    assert z.shape == (C, L // 2 + 1, segments)
    for c in range(C):
        _, _, zr = so.stft(X[c], nperseg=L, noverlap=L - H, complex_output=True)
        assert so.max_rel_err(z[c], zr) <= TOL[dtype]
    torch.cuda.synchronize()


# ------------------------------------------------------ batched / strides ----
@pytest.mark.parametrize("layout", ["rows", "transposed_view", "interleaved"])
def test_batched_layouts(cuda, layout):
    import torch
    C, N, L = 6, 20000, 512
    rng = np.random.default_rng(11)
    X = rng.standard_normal((C, N)).astype(np.float32)
    if layout == "rows":            # (C, N) contiguous, samples along axis 1
        xt, axis = _to_gpu(X, cuda), -1
    elif layout == "transposed_view":  # (N, C) view with strides (1, N)
        xt, axis = _to_gpu(X, cuda).t(), 0
    else:                           # (N, C) contiguous: sample stride C
        xt, axis = _to_gpu(X.T.copy(), cuda), 0
    f, p = ib.spectral(ib.OP_WELCH, xt, nperseg=L, axis=axis, fs=2.0)
    p = _np(p)
    assert p.shape == (C, L // 2 + 1)
    for c in range(C):
        _, pr = so.welch(X[c], fs=2.0, nperseg=L)
        assert so.max_rel_err(p[c], pr) <= 1e-5
    f, t, z = ib.spectral(ib.OP_STFT, xt, nperseg=L, noverlap=384, axis=axis,
                          complex_output=True)
    z = _np(z)
    assert z.shape[:2] == (C, L // 2 + 1)
    for c in (0, C - 1):
        _, _, zr = so.stft(X[c], nperseg=L, noverlap=384, complex_output=True)
        assert so.max_rel_err(z[c], zr) <= 1e-5
    # csd of the same view against a shifted copy
    Y = np.roll(X, 5, axis=1)
    if layout == "rows":
        yt = _to_gpu(Y, cuda)
    elif layout == "transposed_view":
        yt = _to_gpu(Y, cuda).t()
    else:
        yt = _to_gpu(Y.T.copy(), cuda)
    f, pc = ib.spectral(ib.OP_CSD, xt, yt, nperseg=L, axis=axis, complex_output=True)
    pc = _np(pc)
    for c in (0, 3):
        _, pr = so.csd(X[c], Y[c], nperseg=L, complex_output=True)
        assert so.max_rel_err(pc[c], pr) <= 1e-5
    torch.cuda.synchronize()


@pytest.mark.parametrize("complex_output", [True, False])
def test_stft_host_batch_pipelined(cuda, complex_output):
    """Host input and host output of a channel batch: the copies and kernels
    run per channel chunk on several streams."""
    C, N, L = 11, 40000, 1024
    rng = np.random.default_rng(17)
    X = rng.standard_normal((C, N)).astype(np.float32)
    f, t, z = ib.spectral(ib.OP_STFT, X, nperseg=L, noverlap=768,
                          complex_output=complex_output)
    assert isinstance(z, np.ndarray)
    for c in range(C):
        _, _, zr = so.stft(X[c], nperseg=L, noverlap=768,
                           complex_output=complex_output)
        assert so.max_rel_err(z[c], zr) <= 1e-5


def test_storage_offset_view(cuda):
    import torch
    base = _to_gpu(_sig(50000, np.float64, 4), cuda)
    view = base[1234:1234 + 30000:2]          # offset and stride 2
    x = _np(view)
    r = ib.welch(view, nperseg=1024)
    _, p = so.welch(x, nperseg=1024)
    assert so.max_rel_err(_np(r.Pxx), p) <= 1e-12
    torch.cuda.synchronize()


# ---------------------------------------------- segment-range shards + sums ----
@pytest.mark.parametrize("op", ["welch", "csd"])
@pytest.mark.parametrize("dtype", [np.float32, np.float64])
def test_span_shards_scaled_with_the_whole_count(cuda, op, dtype):
    """Each shard holds only its samples and averages over the whole signal's
    segment count (avg_segments): the shards' outputs sum to the PSD."""
    import torch
    from insight_b200 import shard
    L, ov, n = 256, 96, 40 * 256 + 77
    x = _sig(n, dtype, 31)
    y = _sig(n, dtype, 32)
    step, S = shard.framing(n, L, ov)
    code = ib.OP_WELCH if op == "welch" else ib.OP_CSD
    F = L // 2 + 1
    total = None
    for k in range(3):
        s0, s1, lo, hi = shard.segment_shard(n, L, ov, k, 3)
        out = torch.empty(F, dtype=torch.complex128, device=cuda) if op == "csd" else None
        _, part = ib.spectral(code, _to_gpu(x[lo:hi], cuda),
                              _to_gpu(y[lo:hi], cuda) if op == "csd" else None,
                              fs=3.0, window="hamming", nperseg=L, noverlap=ov,
                              seg_range=(0, s1 - s0), avg_segments=S, out=out)
        total = part if total is None else total + part
    torch.cuda.synchronize()
    if op == "welch":
        _, ref = so.welch(x, fs=3.0, window="hamming", nperseg=L, noverlap=ov)
    else:
        _, ref = so.csd(x, y, fs=3.0, window="hamming", nperseg=L, noverlap=ov,
                        complex_output=True)
    tol = 1e-5 if dtype == np.float32 else 1e-12
    assert so.max_rel_err(total.cpu().numpy(), ref) <= tol


def test_avg_segments_rejects_negative(cuda):
    with pytest.raises(RuntimeError, match="avg_segments"):
        ib.spectral(ib.OP_WELCH, _to_gpu(_sig(4096, np.float64, 3), cuda),
                    nperseg=256, avg_segments=-1)
@pytest.mark.parametrize("op", ["welch", "csd"])
@pytest.mark.parametrize("shards", [2, 3])
def test_segment_range_sums(cuda, op, shards):
    import torch
    dtype = np.float64
    L = 512
    x = _sig(60 * L + 100, dtype, 21)
    y = _sig(60 * L + 100, dtype, 22)
    code = ib.OP_WELCH if op == "welch" else ib.OP_CSD
    _, S, F = ib.spectral_shape(code, _to_gpu(x, cuda), nperseg=L)
    total = None
    for k in range(shards):
        s0, s1 = S * k // shards, S * (k + 1) // shards
        _, part = ib.spectral(code, _to_gpu(x, cuda),
                              _to_gpu(y, cuda) if op == "csd" else None,
                              nperseg=L, seg_range=(s0, s1), raw_sums=True)
        total = part if total is None else total + part
    ib.finalize_sums(code, total, S, "float64", nperseg=L)
    torch.cuda.synchronize()
    if op == "welch":
        _, ref = so.welch(x, nperseg=L)
    else:
        _, ref = so.csd(x, y, nperseg=L, complex_output=True)
    assert so.max_rel_err(_np(total), ref) <= 1e-12


# ---------------------------------------------------------- plugin boundary ----
def test_plugin_registry_kernels(cuda):
    """InitPluginGPU registers the kernels; call "welch" through the registry
    signature exactly as the reference core's ops().launch would."""
    import ctypes
    import torch
    from insight_b200 import _abi
    lib = _abi.lib()
    reg = {}

    @_abi.REGISTER_FN
    def register(name, dev, dt, fn):
        reg[(name.decode(), dev, dt)] = fn
        return 0

    iface = _abi.C_DeviceInterface()
    iface.size = ctypes.sizeof(_abi.C_DeviceInterface)
    params = _abi.CustomRuntimeParams()
    params.size = ctypes.sizeof(_abi.CustomRuntimeParams)
    params.interface = ctypes.pointer(iface)
    params.register_kernel = register
    assert lib.InitPluginGPU(ctypes.byref(params)) == 0
    assert params.device_type == b"b200"
    assert (params.version.major, params.version.minor) == (1, 0)
    for name in ("welch", "csd", "coherence", "spectrogram", "stft"):
        for dt in (_abi.DT_F32, _abi.DT_F64):
            assert (name, _abi.DEV_GPU, dt) in reg
    for dt in (_abi.DT_C32, _abi.DT_C64):
        assert ("istft", _abi.DEV_GPU, dt) in reg
    assert iface.device_memory_allocate and iface.get_last_error

    x = _sig(40000, np.float32, 8)
    xt = _to_gpu(x, cuda)
    L = 1024
    win = so.get_window("hann", L)
    scale = so.psd_scale(win.astype(np.float32).astype(np.float64), 1e4, "density")
    out = torch.empty(L // 2 + 1, dtype=torch.float64, device=cuda)
    xa, oa = _abi.from_torch(xt), _abi.from_torch(out)
    wa = _abi.from_numpy(win)
    i64 = lambda v: ctypes.c_int64(v)
    i32 = lambda v: ctypes.c_int32(v)
    vals = [i64(L), i64(L // 2), i64(L), i32(1), i32(1), ctypes.c_double(scale), i64(0)]
    ins = (ctypes.c_void_p * 12)(
        ctypes.addressof(oa), ctypes.addressof(xa), ctypes.addressof(xa),
        ctypes.addressof(wa), *[ctypes.addressof(v) for v in vals], None)
    outs = (ctypes.c_void_p * 2)(ctypes.addressof(oa), None)
    fn = ctypes.cast(reg[("welch", _abi.DEV_GPU, _abi.DT_F32)], _abi.KERNEL_FN)
    assert fn(ins, outs) == 0, _abi.last_error()
    _, p = so.welch(x, fs=1e4, nperseg=L)
    assert so.max_rel_err(_np(out), p) <= 1e-5
    # a bad call fails with a message, never with C_FALLBACK (5)
    bad = (ctypes.c_void_p * 3)(ctypes.addressof(oa), ctypes.addressof(xa), None)
    assert fn(bad, outs) == _abi.C_FAILED
    assert "expected" in _abi.last_error()
    # "coherence" through the registry (same layout as "csd")
    y = (0.5 * np.roll(x, 7) + 0.5 * _sig(40000, np.float32, 9)).astype(np.float32)
    ya = _abi.from_torch(_to_gpu(y, cuda))
    ins = (ctypes.c_void_p * 12)(
        ctypes.addressof(oa), ctypes.addressof(xa), ctypes.addressof(ya),
        ctypes.addressof(wa), *[ctypes.addressof(v) for v in vals], None)
    fn = ctypes.cast(reg[("coherence", _abi.DEV_GPU, _abi.DT_F32)], _abi.KERNEL_FN)
    assert fn(ins, outs) == 0, _abi.last_error()
    _, c = so.coherence(x, y, fs=1e4, nperseg=L)
    assert so.max_rel_err(_np(out), c) <= 1e-5


def test_errors_match_reference(cuda):
    x = _to_gpu(_sig(100, np.float64, 1), cuda)
    with pytest.raises(RuntimeError, match="signal too short for given nperseg"):
        ib.welch(x, nperseg=256)
    with pytest.raises(RuntimeError, match="spectrogram: signal too short"):
        ib.spectrogram(x, nperseg=256)
    with pytest.raises(RuntimeError, match="unknown window name 'nope'"):
        ib.welch(x, nperseg=16, window="nope")


def test_stft_batched_long_units(cuda):
    """A batch large enough that each CTA stores several consecutive tiles of
    a channel (the per-row sector carry between tiles), odd segment count."""
    import torch
    C, N, L, H = 24, (1 << 20) + 265, 2048, 512
    g = torch.Generator(device=cuda)
    g.manual_seed(5)
    x = torch.randn((C, N), generator=g, device=cuda, dtype=torch.float32)
    f, t, z = ib.spectral(ib.OP_STFT, x, nperseg=L, noverlap=L - H,
                          complex_output=True)
    S = (N - L) // H + 1
    assert z.shape == (C, L // 2 + 1, S) and S % 2 == 1
    xs = x.cpu().numpy()
    for c in (0, 11, C - 1):
        _, _, zr = so.stft(xs[c], nperseg=L, noverlap=L - H, complex_output=True)
        assert so.max_rel_err(z[c].cpu().numpy(), zr) <= 1e-5
