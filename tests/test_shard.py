"""Host-side multi-rank logic of insight_b200.shard, on CPU ranks (gloo).

The per-rank steps come from the CPU oracle so the test needs no GPU; what
is tested is the sharding (segment ranges, sample spans with halo, channel
blocks), the cross-rank sum through torch.distributed, and the scale /
one-sided mask with the whole signal's segment count: applied by each rank
before the all-reduce (the default), or once to the reduced raw sums.
"""
import os
import socket
import tempfile

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from insight_b200 import shard
from oracle import spectral_oracle as so


def _oracle_partial(x_span, y_span, *, op, fs, window, nperseg, noverlap, nfft,
                    detrend, return_onesided, scaling, n_seg_local, n_seg_total,
                    stream=None):
    x = x_span.numpy()
    y = y_span.numpy() if y_span is not None else x
    sums, n_seg = so.csd_sums(x, y if op == "csd" else x, nperseg, noverlap, nfft,
                              detrend, window=window, onesided=return_onesided)
    assert n_seg == n_seg_local
    if op == "csd":
        return torch.from_numpy(np.ascontiguousarray(sums).astype(np.complex128))
    return torch.from_numpy(np.ascontiguousarray(sums.real))


def _oracle_finalize(sums, *, op, n_seg, x_dtype, fs, window, nperseg, nfft,
                     return_onesided, scaling, stream=None):
    nfft = nfft or nperseg
    win = so.get_window(window, nperseg)
    F = sums.shape[-1]
    f = so.psd_scale(win, fs, scaling) / n_seg * so.onesided_mask(F, nfft,
                                                                  return_onesided)
    return sums * torch.from_numpy(f)


def _oracle_share(x_span, y_span, *, op, fs, window, nperseg, noverlap, nfft,
                  detrend, return_onesided, scaling, n_seg_local, n_seg_total,
                  stream=None):
    """This rank's sums scaled with the whole signal's segment count (the
    default GPU step's contract): the shares sum to the result."""
    sums = _oracle_partial(x_span, y_span, op=op, fs=fs, window=window,
                           nperseg=nperseg, noverlap=noverlap, nfft=nfft,
                           detrend=detrend, return_onesided=return_onesided,
                           scaling=scaling, n_seg_local=n_seg_local,
                           n_seg_total=n_seg_total)
    return _oracle_finalize(sums, op=op, n_seg=n_seg_total, x_dtype="float64",
                            fs=fs, window=window, nperseg=nperseg, nfft=nfft,
                            return_onesided=return_onesided, scaling=scaling)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out_path, op, kw, prescaled):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        rng = np.random.default_rng(42)
        n = kw["n"]
        x = rng.standard_normal(n)
        y = 0.6 * np.roll(x, 9) + 0.4 * rng.standard_normal(n)
        s0, s1, lo, hi = shard.segment_shard(n, kw["nperseg"], kw["noverlap"], rank,
                                             world)
        res = shard.welch_segment_sharded(
            torch.from_numpy(x[lo:hi].copy()), n, rank=rank, world=world,
            y_span=torch.from_numpy(y[lo:hi].copy()), op=op, fs=kw["fs"],
            window=kw["window"], nperseg=kw["nperseg"], noverlap=kw["noverlap"],
            detrend=kw["detrend"], all_reduce=dist.all_reduce,
            partial=_oracle_share if prescaled else _oracle_partial,
            finalize=None if prescaled else _oracle_finalize)
        if rank == 0:
            np.save(out_path, res.numpy())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("prescaled", [True, False])
@pytest.mark.parametrize("world", [2, 3])
@pytest.mark.parametrize("op", ["welch", "csd"])
def test_segment_sharded_reduction(world, op, prescaled):
    kw = dict(n=50_000, fs=7.0, window="hamming", nperseg=512, noverlap=0,
              detrend="constant")
    with tempfile.TemporaryDirectory() as d:
        out = os.path.join(d, "res.npy")
        mp.spawn(_worker, args=(world, _free_port(), out, op, kw, prescaled),
                 nprocs=world, join=True)
        got = np.load(out)
    rng = np.random.default_rng(42)
    x = rng.standard_normal(kw["n"])
    y = 0.6 * np.roll(x, 9) + 0.4 * rng.standard_normal(kw["n"])
    args = dict(fs=kw["fs"], window=kw["window"], nperseg=kw["nperseg"],
                noverlap=kw["noverlap"], detrend=kw["detrend"])
    if op == "welch":
        _, ref = so.welch(x, **args)
    else:
        _, ref = so.csd(x, y, complex_output=True, **args)
    assert so.max_rel_err(got, ref) <= 1e-12


def test_ranges_cover_everything_once():
    for n, world in [(10, 3), (7, 7), (1000, 8), (262143, 8)]:
        seen = []
        for r in range(world):
            lo, hi = shard.block_range(n, r, world)
            seen.extend(range(lo, hi))
        assert seen == list(range(n))
    n, L, ov = 1 << 20, 8192, 4096
    step, S = shard.framing(n, L, ov)
    spans = [shard.segment_shard(n, L, ov, r, 8) for r in range(8)]
    assert spans[0][0] == 0 and spans[-1][1] == S
    for (a0, a1, lo, hi), (b0, *_) in zip(spans, spans[1:]):
        assert a1 == b0 and hi - lo == (a1 - a0 - 1) * step + L
    assert spans[-1][3] <= n


def test_rejects_more_ranks_than_segments():
    with pytest.raises(ValueError):
        shard.segment_shard(3000, 1024, 0, 0, 8)
