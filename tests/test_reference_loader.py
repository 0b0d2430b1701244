"""The plugin as the reference's own core loads and calls it.

The reference core compiled from its sources (oracle/_ref) loads
libinsight_b200_backend.so with its own loader (ins::load_backend ->
try_load_backend, src/init.cpp:173-236,333-343): it dlopens the file from a
backend search path, calls InitPluginGPU with the core's
insight_register_kernel and installs the device interface the plugin fills.
The kernels are then found with insight_has_kernel and launched with
ops().launch (insight_kernel_launch, src/core/kernel.cpp:199-239) on arrays
the core itself moved to GPUPlace(0) through that device interface: the GPU
branch INTEGRATION.md gives for the frontend, written in
oracle/ref_harness.cpp (ref_gpu_csd, ref_gpu_stft).  Nothing in this file
calls the plugin directly.

The file name sorts after test_oracle.py: once the core has a GPU backend,
later reference calls in the same process would default to the GPU, so the
CPU oracle tests run first (the harness also sets the thread's default place
back to the CPU).
"""
import ctypes
import os
import sys

import numpy as np
import pytest

from oracle import ref_runner
from oracle import spectral_oracle as so

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PLUGIN_DIR = os.path.join(ROOT, "insight_b200")
GOLDEN = os.path.join(ROOT, "tests", "golden")
DT_F32, DT_F64, DT_C32, DT_C64 = 9, 10, 11, 12

needs_ref = pytest.mark.skipif(not ref_runner.available(),
                               reason="oracle/_ref not built")


def _has_gpu():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False


@needs_ref
@pytest.mark.skipif(_has_gpu(), reason="checks the refusal without a GPU")
def test_core_loader_finds_plugin_and_plugin_refuses_without_b200():
    """Without an sm_100 GPU the plugin's InitPluginGPU returns C_FAILED, so
    the core keeps no GPU backend (and never gets a CPU fallback from it)."""
    with pytest.raises(RuntimeError, match="did not load libinsight_b200_backend"):
        ref_runner.load_gpu_backend(PLUGIN_DIR, "b200")
    assert not ref_runner.has_gpu_kernel("welch", DT_F32)


def _launches():
    lib = ctypes.CDLL(os.path.join(PLUGIN_DIR, "libinsight_b200_backend.so"))
    lib.insight_b200_launch_count.restype = ctypes.c_int64
    return lib.insight_b200_launch_count()


def _sig(n, dt, seed):
    rng = np.random.default_rng(seed)
    t = np.arange(n)
    return (rng.standard_normal(n) + np.sin(2 * np.pi * 0.11 * t)).astype(dt)


@needs_ref
@pytest.mark.gpu
def test_core_loads_plugin_and_dispatches_through_its_registry(cuda):
    ref_runner.load_gpu_backend(PLUGIN_DIR, "b200")
    for op in ("welch", "csd", "coherence", "spectrogram", "stft"):
        for dt in (DT_F32, DT_F64):
            assert ref_runner.has_gpu_kernel(op, dt), (op, dt)
    for dt in (DT_C32, DT_C64):
        assert ref_runner.has_gpu_kernel("istft", dt)

    n0 = _launches()
    # welch f32 at the first benchmark configuration, against the reference's
    # own output on the same channel
    sys.path.insert(0, GOLDEN)
    import config_inputs as ci
    g = np.load(os.path.join(GOLDEN, "reference_configs.npz"))
    _, make, _, kw = ci.CASES[0]
    f, p = ref_runner.gpu_csd("welch", make(), **kw)
    assert np.array_equal(f, g["config_1/f"])
    assert so.max_rel_err(p, g["config_1/Pxx"]) <= 1e-5

    # csd and coherence in f64, two-sided welch in f32 with zero padding
    x = _sig(20000, np.float64, 1)
    y = (0.6 * np.roll(x, 5) + 0.4 * _sig(20000, np.float64, 2))
    f, p = ref_runner.gpu_csd("csd", x, y, fs=3.0, window="hamming", nperseg=512)
    _, pr = so.csd(x, y, fs=3.0, window="hamming", nperseg=512)
    assert so.max_rel_err(p, pr) <= 1e-12
    f, c = ref_runner.gpu_csd("coherence", x, y, nperseg=256, noverlap=192)
    _, cr = so.coherence(x, y, nperseg=256, noverlap=192)
    assert so.max_rel_err(c, cr) <= 1e-12
    x32 = _sig(30000, np.float32, 3)
    f, p = ref_runner.gpu_csd("welch", x32, window="blackman", nperseg=300,
                              nfft=512, detrend="none", return_onesided=False,
                              scaling="spectrum")
    fr, pr = so.welch(x32, window="blackman", nperseg=300, nfft=512, detrend="none",
                      return_onesided=False, scaling="spectrum")
    assert np.array_equal(f, fr) and so.max_rel_err(p, pr) <= 1e-5

    # stft f32 at the stft configuration's nperseg / hop: Re(X) (n_freq, n_seg)
    xs = _sig(2048 + 40 * 512, np.float32, 4)
    s = ref_runner.gpu_stft(xs, nperseg=2048, noverlap=1536)
    _, _, z = so.stft(xs, nperseg=2048, noverlap=1536, complex_output=True)
    assert s.shape == z.shape
    assert so.max_rel_err(s, z.real) <= 1e-5

    # every result above came from the plugin's kernels, reached only through
    # the core's registry
    assert _launches() - n0 >= 5
