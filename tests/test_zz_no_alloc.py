"""insight_b200_welch_noalloc: welch without device allocations.

The entry point serves callers that cannot let a library allocate GPU memory:
a host framework that hands out every device buffer from its own pool, or a
latency-critical path that must not pay cudaMalloc/cudaFree's implicit device
synchronisation.  It keeps its working memory in a fixed file-scope device
array instead.  This test calls it through the C ABI twice in a row, on
different shapes and dtypes (so the second call runs over the first call's
leftovers in the shared array), and checks each result against the regular
entry point within the parity tolerances of the other tests (1e-5 for f32,
1e-12 for f64, relative to the largest bin).

The file name sorts last so that a run stopping at the first failure has run
every other test before this one.
"""
import ctypes

import numpy as np
import pytest

import insight_b200 as ib
from insight_b200 import _abi
from oracle import spectral_oracle as so

pytestmark = pytest.mark.gpu


def _noalloc(x, dtype_code, C, N, cs, ss, out, **kw):
    import torch
    lib = _abi.lib()
    status = lib.insight_b200_welch_noalloc(
        ctypes.c_void_p(x.data_ptr()), dtype_code, C, N, cs, ss, kw.get("fs", 1.0),
        kw.get("window", "hann").encode(), kw["nperseg"], kw.get("noverlap", 0),
        kw.get("nfft", 0), kw.get("detrend", "constant").encode(),
        1 if kw.get("return_onesided", True) else 0,
        kw.get("scaling", "density").encode(), ctypes.c_void_p(out.data_ptr()),
        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    return status


def test_noalloc_matches_regular_entry_point_twice(cuda):
    import torch
    torch.cuda.set_device(cuda)
    rng = np.random.default_rng(77)

    # call 1: f32, 8 channels in rows, nperseg 1024
    C, N = 8, 1 << 18
    X = rng.standard_normal((C, N)).astype(np.float32)
    xt = torch.from_numpy(X).to(cuda)
    kw = dict(fs=1e4, nperseg=1024, noverlap=512)
    out = torch.full((C, 513), float("nan"), dtype=torch.float64, device=cuda)
    assert _noalloc(xt, _abi.DT_F32, C, N, N, 1, out, **kw) == 0, _abi.last_error()
    _, ref = ib.spectral(ib.OP_WELCH, xt, **kw)
    assert so.max_rel_err(out.cpu().numpy(), ref.cpu().numpy()) <= 1e-5

    # call 2: f64, one strided channel (every other sample), hamming, 2048
    base = torch.from_numpy(rng.standard_normal(3 << 18)).to(cuda)
    view = base[7::2]
    kw2 = dict(fs=3.0, window="hamming", nperseg=2048, detrend="none",
               scaling="spectrum")
    out2 = torch.full((1025,), float("nan"), dtype=torch.float64, device=cuda)
    ptr = base[7:]  # data_ptr of sample 0 of the view
    assert _noalloc(ptr, _abi.DT_F64, 1, view.shape[0], 0, 2, out2, **kw2) == 0, \
        _abi.last_error()
    ref2 = ib.welch(view, **kw2).Pxx
    assert so.max_rel_err(out2.cpu().numpy(), ref2.cpu().numpy()) <= 1e-12
    assert torch.isfinite(out2).all()


def test_noalloc_near_its_limit_two_sided_and_padded(cuda):
    """Shapes that reach the caps on the work split (1000 channels of 513
    f64 partial-sum bins take most of the 8 MiB array), a two-sided result
    and zero padding, each checked against the regular entry point; after a
    warm-up call, a further call leaves the device's free memory unchanged."""
    import torch
    torch.cuda.set_device(cuda)
    rng = np.random.default_rng(78)
    C, N = 1000, 1 << 14
    xt = torch.from_numpy(rng.standard_normal((C, N)).astype(np.float32)).to(cuda)
    kw = dict(fs=2.0, nperseg=1024)
    out = torch.full((C, 513), float("nan"), dtype=torch.float64, device=cuda)
    assert _noalloc(xt, _abi.DT_F32, C, N, N, 1, out, **kw) == 0, _abi.last_error()
    _, ref = ib.spectral(ib.OP_WELCH, xt, **kw)
    assert so.max_rel_err(out.cpu().numpy(), ref.cpu().numpy()) <= 1e-5

    # two-sided f32, 3 channels
    x3 = xt[:3]
    kw3 = dict(nperseg=512, noverlap=384, return_onesided=False)
    out3 = torch.full((3, 512), float("nan"), dtype=torch.float64, device=cuda)
    assert _noalloc(x3, _abi.DT_F32, 3, N, N, 1, out3, **kw3) == 0, _abi.last_error()
    _, ref3 = ib.spectral(ib.OP_WELCH, x3, **kw3)
    assert so.max_rel_err(out3.cpu().numpy(), ref3.cpu().numpy()) <= 1e-5

    # f32 with zero padding (nfft > nperseg) and no detrend
    kw4 = dict(nperseg=1000, nfft=2048, detrend="none", window="blackman")
    out4 = torch.full((2, 1025), float("nan"), dtype=torch.float64, device=cuda)
    assert _noalloc(xt, _abi.DT_F32, 2, N, N, 1, out4, **kw4) == 0, _abi.last_error()
    _, ref4 = ib.spectral(ib.OP_WELCH, xt[:2], **kw4)
    assert so.max_rel_err(out4.cpu().numpy(), ref4.cpu().numpy()) <= 1e-5

    # no device allocation: the free bytes do not move across a call
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info(cuda)
    assert _noalloc(xt, _abi.DT_F32, C, N, N, 1, out, **kw) == 0, _abi.last_error()
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info(cuda)
    assert free1 == free0
    assert so.max_rel_err(out.cpu().numpy(), ref.cpu().numpy()) <= 1e-5


def test_noalloc_rejects_requests_beyond_its_scratch(cuda):
    import torch
    x = torch.zeros((1024, 8192), dtype=torch.float64, device=cuda)
    out = torch.zeros((1024, 2049), dtype=torch.float64, device=cuda)
    assert _noalloc(x, _abi.DT_F64, 1024, 8192, 8192, 1, out, nperseg=4096) == \
        _abi.C_FAILED
    assert "8 MiB" in _abi.last_error()
