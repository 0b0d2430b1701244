"""Spectral estimation on the B200 backend, with the reference's Python API.

Mirrors ``insight.signal`` (bindings/python/insight/signal/spectral.py:22-118
and bindings/python/insight_py.cpp:1585-1610): same function names, argument
names, defaults and result attributes (``f``, ``Pxx`` / ``f``, ``t``,
``Sxx``).  Every call goes through the C ABI of
``libinsight_b200_backend.so`` (include/insight_b200.h) and runs the fused
sm_100a kernels; nothing here computes a spectrum.

Inputs may be numpy arrays (host memory: the backend copies them to the GPU
and the results come back as numpy arrays, like the reference's CPU
results) or torch tensors on a CUDA device (results are CUDA tensors on the
same device).  2-D inputs are a batch of channels along ``axis``.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Any, Optional

import numpy as np

from . import _abi

__all__ = ["SpectralResult", "SpectrogramResult", "welch", "csd", "coherence",
           "periodogram", "spectrogram", "stft", "istft", "spectral",
           "spectral_shape", "finalize_sums", "SpectralPlan"]


@dataclass
class SpectralResult:
    f: Any
    Pxx: Any


@dataclass
class SpectrogramResult:
    f: Any
    t: Any
    Sxx: Any


def _is_torch(x) -> bool:
    return hasattr(x, "untyped_storage")


def _stream_arg(stream, x):
    """The cudaStream_t of a call: the caller's stream, else, for a CUDA
    tensor input, torch's current stream on its device, so the call is
    ordered after the work that produced the input (the backend's own stream
    would not wait for it); None for host inputs."""
    if stream is None:
        if not (_is_torch(x) and x.is_cuda):
            return None
        import torch
        stream = torch.cuda.current_stream(x.device)
    h = stream if isinstance(stream, int) else stream.cuda_stream
    # NULL selects the backend's own stream in the C ABI; torch's default
    # stream is the legacy NULL stream, named explicitly as cudaStreamLegacy
    return ctypes.c_void_p(h if h else _CUDA_STREAM_LEGACY)


_CUDA_STREAM_LEGACY = 0x1  # cudaStreamLegacy (driver_types.h)


def _inputs_ready(*xs):
    """The reference-signature functions are synchronous and run on the
    backend's stream: let torch's pending work on CUDA inputs finish first."""
    for x in xs:
        if x is not None and _is_torch(x) and x.is_cuda:
            import torch
            torch.cuda.current_stream(x.device).synchronize()
            return


def _empty_like_place(x, shape, dtype: str):
    """Output buffer on x's place: numpy for host inputs, torch on x's device."""
    if _is_torch(x):
        import torch
        tdt = {"float64": torch.float64, "complex64": torch.complex64,
               "complex128": torch.complex128, "float32": torch.float32}[dtype]
        return torch.empty(shape, dtype=tdt, device=x.device)
    return np.empty(shape, dtype=dtype)


_DESC_CACHE: dict = {}


def _desc(op, fs, window, nperseg, noverlap, nfft, detrend, return_onesided,
          scaling="density", mode="psd", axis=-1, seg_range=None, raw_sums=False,
          avg_segments=0):
    """The call descriptor; repeated calls with the same arguments reuse one
    (the backend only reads it)."""
    key = (op, fs, window, nperseg, noverlap, nfft, detrend, return_onesided,
           scaling, mode, axis, seg_range, raw_sums, int(avg_segments or 0))
    d = _DESC_CACHE.get(key)
    if d is None:
        if len(_DESC_CACHE) >= 256:
            _DESC_CACHE.clear()
        d = _DESC_CACHE[key] = _make_desc(*key)
    return d


def _make_desc(op, fs, window, nperseg, noverlap, nfft, detrend, return_onesided,
               scaling, mode, axis, seg_range, raw_sums, avg_segments):
    d = _abi.SpectralDesc()
    d.op = op
    d.axis = axis
    d.fs = float(fs)
    d.window = window.encode()
    d.nperseg = int(nperseg)
    d.noverlap = int(noverlap or 0)
    d.nfft = int(nfft or 0)
    d.detrend = detrend.encode()
    d.return_onesided = 1 if return_onesided else 0
    d.scaling = scaling.encode()
    d.mode = mode.encode()
    d.seg_begin, d.seg_end = (seg_range if seg_range is not None else (0, 0))
    d.raw_sums = 1 if raw_sums else 0
    d.avg_segments = int(avg_segments)
    return d


def spectral_shape(op, x, nperseg=256, noverlap=None, nfft=None,
                   return_onesided=True, axis=-1):
    """(channels, segments, bins) of a call, computed by the backend."""
    d = _desc(op, 1.0, "hann", nperseg, noverlap, nfft, "constant",
              return_onesided, axis=axis)
    xa = _abi.as_array(x)
    c, s, f = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int64()
    _abi.check(_abi.lib().insight_b200_spectral_shape(
        ctypes.byref(d), ctypes.byref(xa), ctypes.byref(c), ctypes.byref(s),
        ctypes.byref(f)), "spectral_shape")
    return c.value, s.value, f.value


def spectral(op, x, y=None, *, fs=1.0, window="hann", nperseg=256, noverlap=None,
             nfft=None, detrend="constant", return_onesided=True,
             scaling="density", mode="psd", axis=-1, complex_output=False,
             seg_range=None, raw_sums=False, avg_segments=0, out=None, stream=None,
             sync=True, axes=True):
    """Native batched entry point (insight_b200_spectral).

    Returns ``(f, out)`` for welch/csd and ``(f, t, out)`` for
    spectrogram/stft.  ``out`` layouts: welch/csd ``[C, F]`` (F64, or
    complex64/complex128 cross spectra with ``complex_output``; raw sums are
    F64 / complex128); spectrogram/stft F64 ``[C, S, F]`` (the reference's
    (n_seg, n_freq) orientation) or complex ``[C, F, S]`` with
    ``complex_output``.  1-D inputs drop the leading channel axis.
    ``avg_segments`` (welch/csd) averages over that many segments instead of
    the call's own count: a shard holding one segment range of a longer
    signal passes the whole signal's count, and the shards' outputs sum to
    the PSD.
    """
    d = _desc(op, fs, window, nperseg, noverlap, nfft, detrend, return_onesided,
              scaling, mode, axis, seg_range, raw_sums, avg_segments)
    xa = _abi.as_array(x)
    ya = _abi.as_array(y) if y is not None else None
    if out is None or axes:
        # geometry is needed only to allocate outputs (a caller-provided out
        # with axes=False skips this host call on the launch path)
        C, S, F = spectral_shape(op, x, nperseg, noverlap, nfft, return_onesided,
                                 axis)
        if op == _abi.OP_STFT:
            F = (int(nfft or nperseg)) // 2 + 1
        s0, s1 = (seg_range if seg_range is not None else (0, S))
        Sl = s1 - s0
    batched = x.ndim == 2
    f32 = str(x.dtype).endswith("float32")
    cdt = "complex64" if f32 else "complex128"
    if out is None:
        if op in (_abi.OP_WELCH, _abi.OP_CSD, _abi.OP_COHERENCE):
            shape = (C, F) if batched else (F,)
            if raw_sums and op == _abi.OP_CSD:
                dt = "complex128"
            elif complex_output and op == _abi.OP_CSD:
                dt = cdt
            else:
                dt = "float64"
        else:
            if complex_output:
                shape = (C, F, Sl) if batched else (F, Sl)
                dt = cdt
            else:
                shape = (C, Sl, F) if batched else (Sl, F)
                dt = "float64"
        out = _empty_like_place(x, shape, dt)
    fo = _empty_like_place(x, (F,), "float64") if axes else None
    oa, fa = _abi.as_array(out), _abi.as_array(fo)
    ta, to = None, None
    if axes and op in (_abi.OP_SPECTROGRAM, _abi.OP_STFT):
        to = _empty_like_place(x, (S,), "float64")
        ta = _abi.as_array(to)
    st = _stream_arg(stream, x)
    _abi.check(_abi.lib().insight_b200_spectral(
        ctypes.byref(d), ctypes.byref(xa), _abi.ptr(ya), ctypes.byref(oa),
        _abi.ptr(fa), _abi.ptr(ta), st, 1 if sync else 0),
        ["welch", "csd", "spectrogram", "stft", "coherence"][op])
    if op in (_abi.OP_WELCH, _abi.OP_CSD, _abi.OP_COHERENCE):
        return fo, out
    return fo, to, out


class SpectralPlan:
    """One ``spectral`` call on fixed CUDA tensors, captured into a CUDA
    graph (insight_b200_plan_create).  ``run()`` replays the call's kernels
    with one graph launch: for loops that repeat the same call on the same
    tensors and would otherwise be bound by per-call host work and launch
    latency (short signals).  Each run recomputes ``out`` from the current
    contents of ``x`` (and ``y``); runs of one plan must not overlap on the
    GPU.  The arguments are those of ``spectral`` (``out`` required, no f /
    t axes)."""

    def __init__(self, op, x, y=None, *, out, fs=1.0, window="hann", nperseg=256,
                 noverlap=None, nfft=None, detrend="constant", return_onesided=True,
                 scaling="density", mode="psd", axis=-1, seg_range=None,
                 raw_sums=False, avg_segments=0, stream=None):
        self._h = None
        d = _desc(op, fs, window, nperseg, noverlap, nfft, detrend, return_onesided,
                  scaling, mode, axis, seg_range, raw_sums, avg_segments)
        xa, ya, oa = _abi.as_array(x), _abi.as_array(y), _abi.as_array(out)
        h = ctypes.c_void_p()
        _abi.check(_abi.lib().insight_b200_plan_create(
            ctypes.byref(d), ctypes.byref(xa), _abi.ptr(ya), ctypes.byref(oa),
            _stream_arg(stream, x), ctypes.byref(h)), "SpectralPlan")
        self._h = h
        self._keep = (x, y, out, d)
        self.out = out

    def run(self, stream=None, sync=False):
        """Launch the captured call on ``stream`` (default: torch's current
        stream of x's device); returns ``out``."""
        _abi.check(_abi.lib().insight_b200_plan_execute(
            self._h, _stream_arg(stream, self._keep[0]), 1 if sync else 0),
            "SpectralPlan.run")
        return self.out

    def close(self):
        if self._h is not None:
            _abi.lib().insight_b200_plan_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def finalize_sums(op, sums, n_seg, x_dtype, *, fs=1.0, window="hann", nperseg=256,
                  nfft=None, return_onesided=True, scaling="density", stream=None):
    """Scale and mask reduced raw welch/csd sums in place (CUDA tensor)."""
    d = _desc(op, fs, window, nperseg, 0, nfft, "constant", return_onesided, scaling)
    sa = _abi.as_array(sums)
    dt = _abi.DT_F32 if str(x_dtype).endswith("float32") else _abi.DT_F64
    st = _stream_arg(stream, sums)
    _abi.check(_abi.lib().insight_b200_finalize_sums(
        ctypes.byref(d), int(n_seg), dt, ctypes.byref(sa), st), "finalize_sums")
    return sums


# ---------------------------------------------------------------------------
# Reference-signature functions (ins.signal.*)
# ---------------------------------------------------------------------------
def _f_out(x, nperseg, nfft, onesided):
    n = int(nfft or nperseg)
    return n // 2 + 1 if onesided else n


def csd(x, y, fs=1.0, window="hann", nperseg=256, noverlap=None, nfft=None,
        detrend="constant", return_onesided=True, scaling="density"):
    """Cross power spectral density (reference csd: real part, F64)."""
    xa, ya = _abi.as_array(x), _abi.as_array(y)
    F = _f_out(x, nperseg, nfft, return_onesided)
    shape = (x.shape[0], F) if x.ndim == 2 else (F,)
    pxy = _empty_like_place(x, shape, "float64")
    f = _empty_like_place(x, (F,), "float64")
    _inputs_ready(x, y)
    _abi.check(_abi.lib().insight_b200_csd(
        ctypes.byref(xa), ctypes.byref(ya), float(fs), window.encode(), int(nperseg),
        int(noverlap or 0), int(nfft or 0), detrend.encode(),
        1 if return_onesided else 0, scaling.encode(), ctypes.byref(_abi.as_array(f)),
        ctypes.byref(_abi.as_array(pxy))), "csd")
    return SpectralResult(f, pxy)


def welch(x, fs=1.0, window="hann", nperseg=256, noverlap=None, nfft=None,
          detrend="constant", return_onesided=True, scaling="density"):
    """Power spectral density by Welch's method (reference welch)."""
    xa = _abi.as_array(x)
    F = _f_out(x, nperseg, nfft, return_onesided)
    shape = (x.shape[0], F) if x.ndim == 2 else (F,)
    pxx = _empty_like_place(x, shape, "float64")
    f = _empty_like_place(x, (F,), "float64")
    _inputs_ready(x)
    _abi.check(_abi.lib().insight_b200_welch(
        ctypes.byref(xa), float(fs), window.encode(), int(nperseg),
        int(noverlap or 0), int(nfft or 0), detrend.encode(),
        1 if return_onesided else 0, scaling.encode(), ctypes.byref(_abi.as_array(f)),
        ctypes.byref(_abi.as_array(pxx))), "welch")
    return SpectralResult(f, pxx)


def coherence(x, y, fs=1.0, window="hann", nperseg=256, noverlap=None, nfft=None,
              detrend="constant"):
    """Magnitude-squared coherence (reference coherence: Re(Pxy)^2 / (Pxx Pyy),
    one pass over x and y)."""
    xa, ya = _abi.as_array(x), _abi.as_array(y)
    F = _f_out(x, nperseg, nfft, True)
    shape = (x.shape[0], F) if x.ndim == 2 else (F,)
    cxy = _empty_like_place(x, shape, "float64")
    f = _empty_like_place(x, (F,), "float64")
    _inputs_ready(x, y)
    _abi.check(_abi.lib().insight_b200_coherence(
        ctypes.byref(xa), ctypes.byref(ya), float(fs), window.encode(), int(nperseg),
        int(noverlap or 0), int(nfft or 0), detrend.encode(),
        ctypes.byref(_abi.as_array(f)), ctypes.byref(_abi.as_array(cxy))),
        "coherence")
    return SpectralResult(f, cxy)


def periodogram(x, fs=1.0, window="boxcar", nfft=None, detrend="constant",
                return_onesided=True, scaling="density"):
    """Reference periodogram: welch with nperseg 256 and the default overlap."""
    xa = _abi.as_array(x)
    F = _f_out(x, 256, nfft, return_onesided)
    shape = (x.shape[0], F) if x.ndim == 2 else (F,)
    pxx = _empty_like_place(x, shape, "float64")
    f = _empty_like_place(x, (F,), "float64")
    _inputs_ready(x)
    _abi.check(_abi.lib().insight_b200_periodogram(
        ctypes.byref(xa), float(fs), window.encode(), int(nfft or 0),
        detrend.encode(), 1 if return_onesided else 0, scaling.encode(),
        ctypes.byref(_abi.as_array(f)), ctypes.byref(_abi.as_array(pxx))),
        "periodogram")
    return SpectralResult(f, pxx)


def istft(Zxx, fs=1.0, window="hann", nperseg=0, noverlap=0, nfft=0, *,
          out=None, stream=None, sync=True):
    """Inverse STFT (reference istft): F64 signal of length
    (n_frames - 1) * hop + nperseg.  Zxx is complex (n_freq, n_frames), or a
    (C, n_freq, n_frames) batch (then the result is (C, n_total)).  fs is
    unused, as in the reference."""
    za = _abi.as_array(Zxx)
    if out is None:
        c, n = ctypes.c_int64(), ctypes.c_int64()
        _abi.check(_abi.lib().insight_b200_istft_shape(
            ctypes.byref(za), int(nperseg or 0), int(noverlap or 0),
            int(nfft or 0), ctypes.byref(c), ctypes.byref(n)), "istft")
        shape = (c.value, n.value) if Zxx.ndim == 3 else (n.value,)
        out = _empty_like_place(Zxx, shape, "float64")
    st = _stream_arg(stream, Zxx)
    _abi.check(_abi.lib().insight_b200_istft_async(
        ctypes.byref(za), window.encode(), int(nperseg or 0), int(noverlap or 0),
        int(nfft or 0), ctypes.byref(_abi.as_array(out)), st, 1 if sync else 0),
        "istft")
    return out


def spectrogram(x, fs=1.0, window="hann", nperseg=256, noverlap=None, nfft=None,
                detrend="constant", return_onesided=True, mode="psd"):
    """Spectrogram (reference spectrogram): Sxx is F64 (n_seg, n_freq)."""
    C, S, F = spectral_shape(_abi.OP_SPECTROGRAM, x, nperseg, noverlap, nfft,
                             return_onesided)
    shape = (C, S, F) if x.ndim == 2 else (S, F)
    sxx = _empty_like_place(x, shape, "float64")
    f = _empty_like_place(x, (F,), "float64")
    t = _empty_like_place(x, (S,), "float64")
    _inputs_ready(x)
    _abi.check(_abi.lib().insight_b200_spectrogram(
        ctypes.byref(_abi.as_array(x)), float(fs), window.encode(), int(nperseg),
        int(noverlap or 0), int(nfft or 0), detrend.encode(),
        1 if return_onesided else 0, mode.encode(), ctypes.byref(_abi.as_array(f)),
        ctypes.byref(_abi.as_array(t)), ctypes.byref(_abi.as_array(sxx))),
        "spectrogram")
    return SpectrogramResult(f, t, sxx)


def stft(x, fs=1.0, window="hann", nperseg=256, noverlap=None, nfft=None,
         complex_output=False):
    """Short-time Fourier transform (reference stft: Re(X), F64 (n_seg, n_freq)).

    ``complex_output=True`` returns the full complex STFT, complex64 for f32
    input (complex128 for f64), laid out (n_freq, n_seg) per channel.
    """
    C, S, F = spectral_shape(_abi.OP_STFT, x, nperseg, noverlap, nfft, True)
    F = int(nfft or nperseg) // 2 + 1
    if complex_output:
        dt = "complex64" if str(x.dtype).endswith("float32") else "complex128"
        shape = (C, F, S) if x.ndim == 2 else (F, S)
    else:
        dt = "float64"
        shape = (C, S, F) if x.ndim == 2 else (S, F)
    z = _empty_like_place(x, shape, dt)
    f = _empty_like_place(x, (F,), "float64")
    t = _empty_like_place(x, (S,), "float64")
    _inputs_ready(x)
    _abi.check(_abi.lib().insight_b200_stft(
        ctypes.byref(_abi.as_array(x)), float(fs), window.encode(), int(nperseg),
        int(noverlap or 0), int(nfft or 0), ctypes.byref(_abi.as_array(f)),
        ctypes.byref(_abi.as_array(t)), ctypes.byref(_abi.as_array(z))), "stft")
    return SpectrogramResult(f, t, z)
