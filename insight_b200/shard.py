"""Multi-GPU sharding of the spectral ops (one process per GPU).

* Channel sharding (batches of channels: stft / welch / csd on many channels):
  each rank takes a contiguous block of channels; there is no collective on
  the data path.
* Segment-range sharding (one very long signal): rank r owns the segments
  [s0, s1) of the whole framing and only the samples they cover,
  [s0*step, (s1-1)*step + nperseg), i.e. its share plus an nperseg - step
  halo.  Each rank computes unscaled F64 sums over its segments, one
  all-reduce (sum) over the ranks combines them, and the scale and one-sided
  mask of the reference csd (src/ops/signal/spectral_analysis.cpp:151-166)
  are applied once to the reduced sums with the whole signal's segment count.

The partial-sum step is a callable so the sharding and reduction logic can
be exercised on CPU ranks (gloo) with any implementation of it; the default
runs the B200 kernels.
"""
from __future__ import annotations

from typing import Callable, Optional, Tuple


def block_range(n: int, rank: int, world: int) -> Tuple[int, int]:
    """Contiguous block [lo, hi) of n items owned by rank (sizes differ by at
    most one)."""
    if world <= 0 or not (0 <= rank < world):
        raise ValueError("rank out of range")
    return n * rank // world, n * (rank + 1) // world


def framing(n_samples: int, nperseg: int, noverlap: int = 0,
            for_spectrogram: bool = False) -> Tuple[int, int]:
    """(step, n_seg) with the reference's defaults (noverlap == 0 means
    nperseg/2 for welch/csd, nperseg/8 for spectrogram/stft)."""
    if noverlap == 0:
        noverlap = nperseg // 8 if for_spectrogram else nperseg // 2
    step = nperseg - noverlap
    if step <= 0:
        raise ValueError("noverlap must be less than nperseg")
    n_seg = (n_samples - nperseg) // step + 1 if n_samples >= nperseg else 0
    return step, n_seg


def segment_shard(n_samples: int, nperseg: int, noverlap: int, rank: int,
                  world: int) -> Tuple[int, int, int, int]:
    """(s0, s1, lo, hi): the segments [s0, s1) of rank and the sample range
    [lo, hi) they read."""
    step, S = framing(n_samples, nperseg, noverlap)
    if S < world:
        raise ValueError("fewer segments than ranks")
    s0, s1 = block_range(S, rank, world)
    return s0, s1, s0 * step, (s1 - 1) * step + nperseg


def _gpu_partial(x_span, y_span, *, op, fs, window, nperseg, noverlap, nfft,
                 detrend, return_onesided, scaling, n_seg_local, stream=None):
    from . import signal
    code = 1 if op == "csd" else 0
    _, sums = signal.spectral(code, x_span, y_span, fs=fs, window=window,
                              nperseg=nperseg, noverlap=noverlap, nfft=nfft,
                              detrend=detrend, return_onesided=return_onesided,
                              scaling=scaling, seg_range=(0, n_seg_local),
                              raw_sums=True, stream=stream, axes=False,
                              sync=stream is None)
    return sums


def _gpu_finalize(sums, *, op, n_seg, x_dtype, fs, window, nperseg, nfft,
                  return_onesided, scaling, stream=None):
    from . import signal
    code = 1 if op == "csd" else 0
    return signal.finalize_sums(code, sums, n_seg, x_dtype, fs=fs, window=window,
                                nperseg=nperseg, nfft=nfft,
                                return_onesided=return_onesided, scaling=scaling,
                                stream=stream)


def welch_segment_sharded(x_span, n_samples: int, *, rank: int, world: int,
                          y_span=None, op: str = "welch", fs: float = 1.0,
                          window: str = "hann", nperseg: int = 256,
                          noverlap: int = 0, nfft: int = 0,
                          detrend: str = "constant", return_onesided: bool = True,
                          scaling: str = "density",
                          all_reduce: Optional[Callable] = None,
                          partial: Callable = _gpu_partial,
                          finalize: Callable = _gpu_finalize, stream=None,
                          on_phase: Optional[Callable[[str], None]] = None):
    """Welch PSD (or csd) of one long signal sharded by segment range.

    x_span (and y_span) hold this rank's samples [lo, hi) of
    segment_shard(n_samples, nperseg, noverlap, rank, world).  Returns the
    reduced, scaled result on every rank.  all_reduce(tensor) sums in place
    over the ranks (torch.distributed.all_reduce by default).  on_phase(name),
    when given, is called after each of the three steps has been enqueued
    ("partial", "all_reduce", "finalize"), e.g. to record a CUDA event on
    the stream between them.
    """
    step, S = framing(n_samples, nperseg, noverlap)
    s0, s1, lo, hi = segment_shard(n_samples, nperseg, noverlap, rank, world)
    if len(x_span) != hi - lo:
        raise ValueError(f"rank {rank}: expected {hi - lo} samples, got {len(x_span)}")
    kw = dict(op=op, fs=fs, window=window, nperseg=nperseg, noverlap=noverlap,
              nfft=nfft, detrend=detrend, return_onesided=return_onesided,
              scaling=scaling)
    sums = partial(x_span, y_span if op == "csd" else None, n_seg_local=s1 - s0,
                   stream=stream, **kw)
    if on_phase is not None:
        on_phase("partial")
    if all_reduce is None:
        import torch.distributed as dist
        all_reduce = dist.all_reduce
    if world > 1:
        if stream is not None:
            # order the collective after the partial sums on their stream
            import torch
            with torch.cuda.stream(stream):
                all_reduce(sums)
        else:
            all_reduce(sums)
    if on_phase is not None:
        on_phase("all_reduce")
    x_dtype = str(x_span.dtype)
    res = finalize(sums, op=op, n_seg=S, x_dtype=x_dtype, fs=fs, window=window,
                   nperseg=nperseg, nfft=nfft, return_onesided=return_onesided,
                   scaling=scaling, stream=stream)
    if on_phase is not None:
        on_phase("finalize")
    return res
