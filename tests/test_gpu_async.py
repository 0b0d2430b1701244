"""Asynchronous native calls (sync=False) on several streams.

A call with GPU inputs and outputs and sync=False only enqueues work on its
stream: constant tables are uploaded with asynchronous copies (other streams
wait on an event, not the host), working buffers grow with stream-ordered
allocation, each stream has its own partial-sum scratch, and the f / t axes
are written by a kernel.  These tests check that such a call returns while
earlier work on another stream is still running, that its own work starts
before that earlier work ends, and that welch calls on two streams at once
both give the right result (they would race on a shared scratch buffer).
"""
import numpy as np
import pytest

import insight_b200 as ib
from oracle import spectral_oracle as so

pytestmark = pytest.mark.gpu


def test_async_call_returns_while_another_stream_runs(cuda):
    import torch
    torch.cuda.set_device(cuda)
    sa, sb = torch.cuda.Stream(cuda), torch.cuda.Stream(cuda)
    g = torch.Generator(device=cuda)
    g.manual_seed(11)
    C, N, L, H = 64, 1 << 22, 2048, 512
    S = (N - L) // H + 1
    x = torch.randn((C, N), generator=g, device=cuda)
    za = torch.empty((C, L // 2 + 1, S), dtype=torch.complex64, device=cuda)
    # B: a window, length and padding no earlier test uses (fresh tables) on a
    # stream that has no scratch yet; the f axis is written on the device
    xb = torch.randn((8, 1 << 18), generator=g, device=cuda)
    pb = torch.empty((8, 1025), dtype=torch.float64, device=cuda)
    kwb = dict(fs=7.0, window="nuttall", nperseg=1999, noverlap=1000, nfft=2048)
    # CUDA loads each kernel on its first launch in a process (lazy module
    # loading), which may synchronise the context: run both kernel shapes
    # once first (B's with another window, on another stream, so its tables
    # and its stream's scratch are still new in the timed call)
    warm = torch.cuda.Stream(cuda)
    ib.spectral(ib.OP_STFT, x[:2], complex_output=True, nperseg=L, noverlap=L - H,
                stream=warm)
    ib.spectral(ib.OP_WELCH, xb, stream=warm, axes=True,
                **dict(kwb, window="hann"))
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
    torch.cuda.synchronize()
    ev[0].record(sa)
    for _ in range(3):  # several ms of work on stream A
        ib.spectral(ib.OP_STFT, x, out=za, complex_output=True, nperseg=L,
                    noverlap=L - H, stream=sa, sync=False, axes=False)
    ev[1].record(sa)
    ev[2].record(sb)
    f, _ = ib.spectral(ib.OP_WELCH, xb, out=pb, stream=sb, sync=False, axes=True,
                       **kwb)
    ev[3].record(sb)
    a_pending = not ev[1].query()  # A still running when B's call returned
    torch.cuda.synchronize()
    assert a_pending, "the call on stream B waited for stream A"
    assert ev[0].elapsed_time(ev[2]) < ev[0].elapsed_time(ev[1])
    xh = xb.cpu().numpy()
    for c in (0, 7):
        fr, pr = so.welch(xh[c], **kwb)
        assert so.max_rel_err(pb[c].cpu().numpy(), pr) <= 1e-5
    assert np.array_equal(f.cpu().numpy(), fr)


def test_welch_on_two_streams_at_once(cuda):
    """Two welch calls with sync=False on two streams, enqueued back to back
    with different shapes: each uses its own stream's scratch."""
    import torch
    torch.cuda.set_device(cuda)
    s1, s2 = torch.cuda.Stream(cuda), torch.cuda.Stream(cuda)
    g = torch.Generator(device=cuda)
    g.manual_seed(12)
    x1 = torch.randn((96, 1 << 17), generator=g, device=cuda)
    x2 = torch.randn((40, 1 << 18), generator=g, device=cuda, dtype=torch.float64)
    p1 = torch.empty((96, 513), dtype=torch.float64, device=cuda)
    p2 = torch.empty((40, 2049), dtype=torch.float64, device=cuda)
    torch.cuda.synchronize()
    for _ in range(2):
        ib.spectral(ib.OP_WELCH, x1, out=p1, nperseg=1024, stream=s1, sync=False,
                    axes=False)
        ib.spectral(ib.OP_WELCH, x2, out=p2, nperseg=4096, window="hamming",
                    stream=s2, sync=False, axes=False)
    torch.cuda.synchronize()
    h1, h2 = x1.cpu().numpy(), x2.cpu().numpy()
    for c in (0, 95):
        _, r = so.welch(h1[c], nperseg=1024)
        assert so.max_rel_err(p1[c].cpu().numpy(), r) <= 1e-5
    for c in (0, 39):
        _, r = so.welch(h2[c], nperseg=4096, window="hamming")
        assert so.max_rel_err(p2[c].cpu().numpy(), r) <= 1e-12
