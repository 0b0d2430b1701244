"""insight_b200 — B200-native spectral estimation backend for Insight.

Hot path: the reference's ``signal::welch``, ``signal::csd``,
``signal::spectrogram`` and ``signal::stft`` (and the compositions
``coherence`` and ``periodogram``, and the inverse ``istft``) as one fused
sm_100a kernel family behind
Insight's device-plugin C ABI (include/insight_b200.h).
"""
from . import _abi  # noqa: F401
from .signal import (SpectralPlan, SpectralResult, SpectrogramResult,  # noqa: F401
                     coherence, csd, finalize_sums, istft, periodogram, spectral,
                     spectral_shape, spectrogram, stft, welch)

OP_WELCH = _abi.OP_WELCH
OP_CSD = _abi.OP_CSD
OP_SPECTROGRAM = _abi.OP_SPECTROGRAM
OP_STFT = _abi.OP_STFT
OP_COHERENCE = _abi.OP_COHERENCE


def library_path() -> str:
    return _abi.LIB_PATH


def launch_count() -> int:
    """Kernel launches issued by the backend in this process."""
    return _abi.launch_count()
