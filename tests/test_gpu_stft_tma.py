"""The TMA-store stft kernel (f32, nperseg = nfft = 2048) at its edges.

Its output leaves shared memory in boxes of 8 columns x 256 bin rows, one
tensor map per class of rows R = c*F + k with the same 32-byte phase, with
columns carried between the tiles of a run and stored directly at run and
channel ends.  These cases vary what decides that tiling: the row stride
(phase pattern), channel and segment counts (runs that start and end
mid-channel, single-tile channels), the hop (register reuse of segment b),
and the DC detrend; padding columns and a guard after the output must stay
untouched.  The reference is the CPU oracle, at the f32 bar of 1e-5 of the
max bin.
"""
import numpy as np
import pytest

import insight_b200 as ib
from oracle import spectral_oracle as so

pytestmark = pytest.mark.gpu

L = 2048
F = L // 2 + 1


def _signals(C, N, seed):
    rng = np.random.default_rng(seed)
    t = np.arange(N)
    X = rng.standard_normal((C, N)) + np.sin(2 * np.pi * 0.07 * t)
    return X.astype(np.float32)


def _run(x, hop, detrend, out=None):
    """Complex spectrogram (the stft op with the detrend option)."""
    return ib.spectral(ib.OP_SPECTROGRAM, x, nperseg=L, noverlap=L - hop,
                       detrend=detrend, mode="complex", complex_output=True,
                       out=out)[2]


def _check(z, X, hop, detrend):
    for c in range(X.shape[0]):
        _, _, zr = so.spectrogram(X[c], nperseg=L, noverlap=L - hop,
                                  detrend=detrend, mode="complex",
                                  complex_output=True)
        assert so.max_rel_err(z[c], zr) <= 1e-5, f"channel {c}"


@pytest.mark.parametrize("hop", [512, 1024, 700])
@pytest.mark.parametrize("C,S", [(1, 1), (3, 2), (2, 8), (5, 9), (4, 65),
                                 (7, 300), (1, 1201)])
@pytest.mark.parametrize("pad", [0, 1, 2, 3, 6])
def test_row_strides_and_counts(cuda, hop, C, S, pad):
    """Row stride S + pad (every phase pattern mod 4), padding columns and a
    guard region after the last row filled with NaN and left untouched."""
    import torch
    N = L + (S - 1) * hop + 3
    X = _signals(C, N, 100 + C * 7 + S)
    x = torch.from_numpy(X).to(cuda)
    guard = 4096
    buf = torch.full((C * F * (S + pad) + guard,), float("nan"),
                     dtype=torch.complex64, device=cuda)
    out = buf[: C * F * (S + pad)].view(C, F, S + pad)[:, :, :S]
    _run(x, hop, "none", out)
    z = out.cpu().numpy()
    assert np.isfinite(z).all()
    _check(z, X, hop, "none")
    full = buf.cpu().numpy()
    assert np.isnan(full[C * F * (S + pad):].real).all(), "guard overwritten"
    if pad:
        padcols = full[: C * F * (S + pad)].reshape(C, F, S + pad)[:, :, S:]
        assert np.isnan(padcols.real).all(), "padding columns overwritten"


@pytest.mark.parametrize("detrend", ["constant", "none"])
def test_many_runs_across_channels(cuda, detrend):
    """More tiles than CTAs with runs that start and end mid-channel: 10
    channels of 3001 segments over every SM, hop 512."""
    import torch
    C, S, hop = 10, 3001, 512
    N = L + (S - 1) * hop
    X = _signals(C, N, 77)
    x = torch.from_numpy(X).to(cuda)
    z = _run(x, hop, detrend)
    _check(z.cpu().numpy(), X, hop, detrend)


def test_unaligned_output_falls_back(cuda):
    """An output whose base is not 32-byte aligned takes the other kernel; the
    result is the same."""
    import torch
    C, S, hop = 3, 40, 512
    N = L + (S - 1) * hop
    X = _signals(C, N, 5)
    x = torch.from_numpy(X).to(cuda)
    buf = torch.empty(C * F * S + 1, dtype=torch.complex64, device=cuda)
    out = buf[1:].view(C, F, S)
    _run(x, hop, "constant", out)
    _check(out.cpu().numpy(), X, hop, "constant")


def test_two_calls_same_buffer(cuda):
    """Back-to-back calls into the same output with different inputs: nothing
    of the first call survives in the second's result."""
    import torch
    C, S, hop = 4, 129, 1024
    N = L + (S - 1) * hop
    X1, X2 = _signals(C, N, 1), _signals(C, N, 2)
    out = torch.empty((C, F, S), dtype=torch.complex64, device=cuda)
    for X in (X1, X2):
        _run(torch.from_numpy(X).to(cuda), hop, "constant", out)
    _check(out.cpu().numpy(), X2, hop, "constant")
