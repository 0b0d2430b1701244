"""Multi-GPU sharding of the spectral ops (one process per GPU).

* Channel sharding (batches of channels: stft / welch / csd on many channels):
  each rank takes a contiguous block of channels; there is no collective on
  the data path.
* Segment-range sharding (one very long signal): rank r owns the segments
  [s0, s1) of the whole framing and only the samples they cover,
  [s0*step, (s1-1)*step + nperseg), i.e. its share plus an nperseg - step
  halo.  Each rank sums its segments' spectra in F64 and applies the scale
  and one-sided mask of the reference csd
  (src/ops/signal/spectral_analysis.cpp:151-166) with the WHOLE signal's
  segment count (both are linear), so one all-reduce (sum) over the ranks
  leaves the PSD itself on every rank: the collective is the last step.

The per-rank step is a callable so the sharding and reduction logic can be
exercised on CPU ranks (gloo) with any implementation of it; the default
runs the B200 kernels.  A caller may instead return unscaled sums and pass a
finalize callable that scales the reduced sums.
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
                 detrend, return_onesided, scaling, n_seg_local, n_seg_total,
                 stream=None):
    """This rank's share of the result: its segments averaged with the whole
    signal's count (welch F64; csd complex128 cross spectra)."""
    from . import signal
    code = 1 if op == "csd" else 0
    out = None
    if op == "csd":
        import torch
        F = (int(nfft or nperseg) // 2 + 1) if return_onesided else int(nfft or nperseg)
        out = torch.empty(F, dtype=torch.complex128, device=x_span.device)
    _, part = signal.spectral(code, x_span, y_span, fs=fs, window=window,
                              nperseg=nperseg, noverlap=noverlap, nfft=nfft,
                              detrend=detrend, return_onesided=return_onesided,
                              scaling=scaling, seg_range=(0, n_seg_local),
                              avg_segments=n_seg_total, out=out, stream=stream,
                              axes=False, sync=stream is None)
    return part


def welch_segment_sharded(x_span, n_samples: int, *, rank: int, world: int,
                          y_span=None, op: str = "welch", fs: float = 1.0,
                          window: str = "hann", nperseg: int = 256,
                          noverlap: int = 0, nfft: int = 0,
                          detrend: str = "constant", return_onesided: bool = True,
                          scaling: str = "density",
                          all_reduce: Optional[Callable] = None,
                          partial: Callable = _gpu_partial,
                          finalize: Optional[Callable] = None, stream=None,
                          on_phase: Optional[Callable[[str], None]] = None):
    """Welch PSD (or csd) of one long signal sharded by segment range.

    x_span (and y_span) hold this rank's samples [lo, hi) of
    segment_shard(n_samples, nperseg, noverlap, rank, world).  Returns the
    reduced, scaled result on every rank.  all_reduce(tensor) sums in place
    over the ranks (torch.distributed.all_reduce by default).  partial(...)
    returns this rank's share, already averaged over n_seg_total segments,
    unless a finalize(sums, ...) callable is given to scale the reduced sums.
    on_phase(name), when given, is called after each step has been enqueued
    ("partial", "all_reduce", and "finalize" even when there is none), e.g.
    to record a CUDA event on the stream between them.
    """
    step, S = framing(n_samples, nperseg, noverlap)
    s0, s1, lo, hi = segment_shard(n_samples, nperseg, noverlap, rank, world)
    if len(x_span) != hi - lo:
        raise ValueError(f"rank {rank}: expected {hi - lo} samples, got {len(x_span)}")
    kw = dict(op=op, fs=fs, window=window, nperseg=nperseg, noverlap=noverlap,
              nfft=nfft, detrend=detrend, return_onesided=return_onesided,
              scaling=scaling)
    sums = partial(x_span, y_span if op == "csd" else None, n_seg_local=s1 - s0,
                   n_seg_total=S, stream=stream, **kw)
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
    res = sums
    if finalize is not None:
        res = finalize(sums, op=op, n_seg=S, x_dtype=str(x_span.dtype), fs=fs,
                       window=window, nperseg=nperseg, nfft=nfft,
                       return_onesided=return_onesided, scaling=scaling,
                       stream=stream)
    if on_phase is not None:
        on_phase("finalize")
    return res


class SegmentShardPlan:
    """welch_segment_sharded for repeated calls on the same span tensors (a
    signal buffer refilled in place between calls): this rank's step (the
    accumulate kernel and the slot fold, averaged with the whole signal's
    segment count) is captured once into a CUDA graph (signal.SpectralPlan),
    so a call is one graph launch plus the all-reduce.  run() returns the
    reduced result (the same tensor every call)."""

    def __init__(self, x_span, n_samples: int, *, rank: int, world: int,
                 y_span=None, op: str = "welch", fs: float = 1.0,
                 window: str = "hann", nperseg: int = 256, noverlap: int = 0,
                 nfft: int = 0, detrend: str = "constant",
                 return_onesided: bool = True, scaling: str = "density",
                 stream=None):
        import torch

        from . import signal
        _, S = framing(n_samples, nperseg, noverlap)
        s0, s1, lo, hi = segment_shard(n_samples, nperseg, noverlap, rank, world)
        if len(x_span) != hi - lo:
            raise ValueError(f"rank {rank}: expected {hi - lo} samples, "
                             f"got {len(x_span)}")
        n = int(nfft or nperseg)
        F = n // 2 + 1 if return_onesided else n
        csd = op == "csd"
        self.out = torch.empty(F, dtype=torch.complex128 if csd else torch.float64,
                               device=x_span.device)
        self.world, self.stream = world, stream
        self._plan = signal.SpectralPlan(
            signal._abi.OP_CSD if csd else signal._abi.OP_WELCH, x_span,
            y_span if csd else None, out=self.out, fs=fs, window=window,
            nperseg=nperseg, noverlap=noverlap, nfft=nfft, detrend=detrend,
            return_onesided=return_onesided, scaling=scaling,
            seg_range=(0, s1 - s0), avg_segments=S, stream=stream)

    def run(self, all_reduce: Optional[Callable] = None,
            on_phase: Optional[Callable[[str], None]] = None):
        self._plan.run(stream=self.stream)
        if on_phase is not None:
            on_phase("partial")
        if self.world > 1:
            if all_reduce is None:
                import torch.distributed as dist
                all_reduce = dist.all_reduce
            import torch
            with torch.cuda.stream(self.stream):
                all_reduce(self.out)
        if on_phase is not None:
            on_phase("all_reduce")
            on_phase("finalize")
        return self.out

    def close(self):
        self._plan.close()
