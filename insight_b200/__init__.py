"""insight_b200 — B200-native spectral estimation backend for Insight.

Hot path: the reference's ``signal::welch``, ``signal::csd``,
``signal::spectrogram`` and ``signal::stft`` as one fused sm_100a kernel
family behind Insight's device-plugin C ABI (include/insight_b200.h).
"""
from . import _abi  # noqa: F401
from .signal import (SpectralResult, SpectrogramResult, csd, finalize_sums,  # noqa: F401
                     spectral, spectral_shape, spectrogram, stft, welch)

OP_WELCH = _abi.OP_WELCH
OP_CSD = _abi.OP_CSD
OP_SPECTROGRAM = _abi.OP_SPECTROGRAM
OP_STFT = _abi.OP_STFT


def library_path() -> str:
    return _abi.LIB_PATH


def launch_count() -> int:
    """Kernel launches issued by the backend in this process."""
    return _abi.launch_count()
