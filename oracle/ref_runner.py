"""ctypes wrapper of the reference built from its sources (oracle/_ref).

Test infrastructure only: runs the reference's own ins::signal::welch / csd /
spectrogram / stft (src/ops/signal/spectral_analysis.cpp) through
oracle/ref_harness.cpp.  The reference's CPU "fft" kernel exists only with
FFTW3, which is absent here; the harness registers a substitute FFT kernel
through the reference's insight_register_kernel C ABI (see ref_harness.cpp).
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

from .spectral_oracle import framing

HERE = os.path.dirname(os.path.abspath(__file__))
REF_DIR = os.path.join(HERE, "_ref")
HARNESS = os.path.join(REF_DIR, "libinsight_ref_harness.so")

_lib = None


def available() -> bool:
    return os.path.exists(HARNESS) and os.path.exists(
        os.path.join(REF_DIR, "libinsight_cpu_backend.so"))


def lib():
    global _lib
    if _lib is None:
        if not available():
            raise RuntimeError("oracle/_ref is not built (make -C oracle ref)")
        L = ctypes.CDLL(HARNESS, mode=ctypes.RTLD_GLOBAL)
        L.ref_last_error.restype = ctypes.c_char_p
        L.ref_init.argtypes = [ctypes.c_char_p]
        P = ctypes.POINTER(ctypes.c_double)
        I = ctypes.c_int64
        L.ref_csd.argtypes = [ctypes.c_void_p, ctypes.c_void_p, I, ctypes.c_int,
                              ctypes.c_double, ctypes.c_char_p, I, I, I,
                              ctypes.c_char_p, ctypes.c_int, ctypes.c_char_p, P, P, I,
                              ctypes.POINTER(I)]
        L.ref_coherence.argtypes = [ctypes.c_void_p, ctypes.c_void_p, I, ctypes.c_int,
                                    ctypes.c_int, ctypes.c_double, ctypes.c_char_p, I,
                                    I, I, ctypes.c_char_p, ctypes.c_int,
                                    ctypes.c_char_p, P, P, I, ctypes.POINTER(I)]
        L.ref_istft.argtypes = [P, I, I, ctypes.c_char_p, I, I, I, P, I,
                                ctypes.POINTER(I)]
        L.ref_spectrogram.argtypes = [ctypes.c_void_p, I, ctypes.c_int, ctypes.c_double,
                                      ctypes.c_char_p, I, I, I, ctypes.c_char_p,
                                      ctypes.c_int, ctypes.c_char_p, ctypes.c_int, P, P,
                                      P, I, ctypes.POINTER(I), ctypes.POINTER(I)]
        L.ref_set_threads.argtypes = [ctypes.c_int]
        L.ref_set_threads.restype = ctypes.c_int
        if L.ref_init(REF_DIR.encode()) != 0:
            raise RuntimeError("ref_init: " + L.ref_last_error().decode())
        _lib = L
    return _lib


def set_threads(n: int) -> int:
    """Use n OpenMP threads in the reference's loops; returns the count."""
    return int(lib().ref_set_threads(int(n)))


def _dt(x):
    return 9 if x.dtype == np.float32 else 10


def csd(x, y=None, fs=1.0, window="hann", nperseg=256, noverlap=0, nfft=0,
        detrend="constant", return_onesided=True, scaling="density"):
    """Reference csd (y given) or welch (y None): returns (f, Pxx) F64."""
    L = lib()
    x = np.ascontiguousarray(x)
    if y is not None:
        y = np.ascontiguousarray(y, dtype=x.dtype)
    cap = (nfft or nperseg) + 2
    f = np.zeros(cap)
    p = np.zeros(cap)
    nf = ctypes.c_int64()
    P = ctypes.POINTER(ctypes.c_double)
    rc = L.ref_csd(x.ctypes.data, None if y is None else y.ctypes.data, len(x), _dt(x),
                   fs, window.encode(), nperseg, noverlap, nfft, detrend.encode(),
                   1 if return_onesided else 0, scaling.encode(),
                   f.ctypes.data_as(P), p.ctypes.data_as(P), cap, ctypes.byref(nf))
    if rc != 0:
        raise RuntimeError(L.ref_last_error().decode())
    return f[:nf.value].copy(), p[:nf.value].copy()


def welch(x, **kw):
    return csd(x, None, **kw)


def _coh(mode, x, y, fs, window, nperseg, noverlap, nfft, detrend, onesided,
         scaling):
    L = lib()
    x = np.ascontiguousarray(x)
    yp = None
    if y is not None:
        y = np.ascontiguousarray(y, dtype=x.dtype)
        yp = y.ctypes.data
    cap = (nfft or nperseg) + 2
    f = np.zeros(cap)
    p = np.zeros(cap)
    nf = ctypes.c_int64()
    P = ctypes.POINTER(ctypes.c_double)
    rc = L.ref_coherence(x.ctypes.data, yp, len(x), _dt(x), mode, fs,
                         window.encode(), nperseg, noverlap, nfft, detrend.encode(),
                         1 if onesided else 0, scaling.encode(), f.ctypes.data_as(P),
                         p.ctypes.data_as(P), cap, ctypes.byref(nf))
    if rc != 0:
        raise RuntimeError(L.ref_last_error().decode())
    return f[:nf.value].copy(), p[:nf.value].copy()


def coherence(x, y, fs=1.0, window="hann", nperseg=256, noverlap=0, nfft=0,
              detrend="constant"):
    """Reference coherence: returns (f, Cxy) F64."""
    return _coh(1, x, y, fs, window, nperseg, noverlap, nfft, detrend, True,
                "density")


def periodogram(x, fs=1.0, window="boxcar", nfft=0, detrend="constant",
                return_onesided=True, scaling="density"):
    """Reference periodogram (welch with nperseg 256): returns (f, Pxx) F64."""
    return _coh(2, x, None, fs, window, 256, 0, nfft, detrend, return_onesided,
                scaling)


def istft(Zxx, fs=1.0, window="hann", nperseg=0, noverlap=0, nfft=0):
    """Reference istft of a complex (n_freq, n_frames) array: F64 signal."""
    L = lib()
    z = np.ascontiguousarray(Zxx, dtype=np.complex128)
    F, S = z.shape
    nf_ = nfft if nfft > 0 else 2 * (F - 1)
    nps = nperseg if nperseg > 0 else nf_
    cap = (S + 1) * nps + nf_ + 16
    out = np.zeros(cap)
    n = ctypes.c_int64()
    P = ctypes.POINTER(ctypes.c_double)
    rc = L.ref_istft(z.view(np.float64).ctypes.data_as(P), F, S, window.encode(),
                     nperseg, noverlap, nfft, out.ctypes.data_as(P), cap,
                     ctypes.byref(n))
    if rc != 0:
        raise RuntimeError(L.ref_last_error().decode())
    return out[:n.value].copy()


def spectrogram(x, fs=1.0, window="hann", nperseg=256, noverlap=0, nfft=0,
                detrend="constant", return_onesided=True, mode="psd", is_stft=False):
    """Reference spectrogram / stft: returns (f, t, Sxx) with Sxx (n_seg, n_freq)."""
    L = lib()
    x = np.ascontiguousarray(x)
    n = len(x)
    nf_ = nfft or nperseg
    _, S0 = framing(n, nperseg, noverlap, for_spectrogram=True)
    F0 = nf_ // 2 + 1 if return_onesided else nf_
    cap = max(S0 * F0, 1)
    f = np.zeros(F0 + 1)
    t = np.zeros(S0 + 1)
    s = np.zeros(cap)
    ns, nf = ctypes.c_int64(), ctypes.c_int64()
    P = ctypes.POINTER(ctypes.c_double)
    rc = L.ref_spectrogram(x.ctypes.data, n, _dt(x), fs, window.encode(), nperseg,
                           noverlap, nfft, detrend.encode(), 1 if return_onesided else 0,
                           mode.encode(), 1 if is_stft else 0, f.ctypes.data_as(P),
                           t.ctypes.data_as(P), s.ctypes.data_as(P), cap,
                           ctypes.byref(ns), ctypes.byref(nf))
    if rc != 0:
        raise RuntimeError(L.ref_last_error().decode())
    S, F = ns.value, nf.value
    return f[:F].copy(), t[:S].copy(), s[:S * F].reshape(S, F).copy()


def stft(x, fs=1.0, window="hann", nperseg=256, noverlap=0, nfft=0):
    return spectrogram(x, fs, window, nperseg, noverlap, nfft, is_stft=True)


# ---------------------------------------------------------------------------
# The B200 plugin through the reference's own core (loader, registry, Array).
# ---------------------------------------------------------------------------
def load_gpu_backend(search_dir: str, name: str = "b200") -> None:
    """ins::load_backend(name) with search_dir added to the core's backend
    search paths: the core dlopens libinsight_<name>_backend.so, calls its
    InitPluginGPU and installs its device interface.  Raises with the core's
    message when the plugin is not accepted."""
    L = lib()
    L.ref_load_gpu_backend.argtypes = [ctypes.c_char_p, ctypes.c_char_p]
    if L.ref_load_gpu_backend(search_dir.encode(), name.encode()) != 0:
        raise RuntimeError(L.ref_last_error().decode())


def has_gpu_kernel(op: str, dtype_code: int) -> bool:
    """insight_has_kernel(op, GPU, dtype) of the core's registry."""
    L = lib()
    L.ref_has_gpu_kernel.argtypes = [ctypes.c_char_p, ctypes.c_int]
    return bool(L.ref_has_gpu_kernel(op.encode(), dtype_code))


def gpu_csd(op, x, y=None, fs=1.0, window="hann", nperseg=256, noverlap=0,
            nfft=0, detrend="constant", return_onesided=True, scaling="density"):
    """The frontend's GPU branch of csd / welch / coherence run by the core:
    inputs moved to GPUPlace(0) by Array::to, output allocated by the core,
    the registered kernel launched by ops().launch.  Returns (f, P)."""
    L = lib()
    x = np.ascontiguousarray(x)
    if y is not None:
        y = np.ascontiguousarray(y, dtype=x.dtype)
    I = ctypes.c_int64
    P = ctypes.POINTER(ctypes.c_double)
    L.ref_gpu_csd.argtypes = [ctypes.c_char_p, ctypes.c_void_p, ctypes.c_void_p, I,
                              ctypes.c_int, ctypes.c_double, ctypes.c_char_p, I, I,
                              I, ctypes.c_char_p, ctypes.c_int, ctypes.c_char_p, P,
                              P, I, ctypes.POINTER(I)]
    cap = (nfft or nperseg) + 2
    f = np.zeros(cap)
    p = np.zeros(cap)
    nf = I()
    rc = L.ref_gpu_csd(op.encode(), x.ctypes.data, None if y is None else y.ctypes.data,
                       len(x), _dt(x), fs, window.encode(), nperseg, noverlap, nfft,
                       detrend.encode(), 1 if return_onesided else 0,
                       scaling.encode(), f.ctypes.data_as(P), p.ctypes.data_as(P),
                       cap, ctypes.byref(nf))
    if rc != 0:
        raise RuntimeError(L.ref_last_error().decode())
    return f[:nf.value].copy(), p[:nf.value].copy()


def gpu_stft(x, window="hann", nperseg=256, noverlap=0, nfft=0):
    """The frontend's GPU branch of stft run by the core: Re(X) as the
    (n_freq, n_seg) F64 buffer the reference builds, written by the
    registered "stft" kernel."""
    L = lib()
    x = np.ascontiguousarray(x)
    I = ctypes.c_int64
    P = ctypes.POINTER(ctypes.c_double)
    L.ref_gpu_stft.argtypes = [ctypes.c_void_p, I, ctypes.c_int, ctypes.c_double,
                               ctypes.c_char_p, I, I, I, P, I, ctypes.POINTER(I),
                               ctypes.POINTER(I)]
    _, S0 = framing(len(x), nperseg, noverlap, for_spectrogram=True)
    F0 = (nfft or nperseg) // 2 + 1
    s = np.zeros(max(S0 * F0, 1))
    ns, nf = I(), I()
    rc = L.ref_gpu_stft(x.ctypes.data, len(x), _dt(x), 1.0, window.encode(), nperseg,
                        noverlap, nfft, s.ctypes.data_as(P), s.size, ctypes.byref(ns),
                        ctypes.byref(nf))
    if rc != 0:
        raise RuntimeError(L.ref_last_error().decode())
    return s[:nf.value * ns.value].reshape(nf.value, ns.value).copy()
