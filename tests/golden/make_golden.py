"""Generate the golden fixtures from the reference itself.

Runs the reference's own ins::signal::welch / csd / spectrogram / stft,
compiled from its sources into oracle/_ref (``make -C oracle ref``), on small
seeded inputs and stores inputs and outputs in tests/golden/reference_cases.npz.
Also records the C ABI layout of the reference's headers
(include/insight/c_api/*.h) in tests/golden/abi_layout.json.

    python tests/golden/make_golden.py <reference source tree>

The fixtures are committed; the tests never need the reference tree.
"""
from __future__ import annotations

import json
import os
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import ref_runner  # noqa: E402
from oracle import spectral_oracle as so  # noqa: E402

# (name, op, dtype, n, kwargs)
CASES = [
    ("welch_f64_hann", "welch", "f64", 4000, dict(fs=1e4, nperseg=256)),
    ("welch_f64_hamming_pad", "welch", "f64", 3000,
     dict(fs=2.0, window="hamming", nperseg=100, nfft=128)),
    ("welch_f64_blackman_none_twosided", "welch", "f64", 2500,
     dict(window="blackman", nperseg=64, detrend="none", return_onesided=False,
          scaling="spectrum")),
    ("welch_f64_linear_is_none", "welch", "f64", 3000,
     dict(nperseg=128, detrend="linear")),
    ("welch_f64_overlap", "welch", "f64", 5001, dict(nperseg=256, noverlap=200)),
    ("welch_f32_promoted", "welch", "f32", 4096, dict(fs=1e4, nperseg=1024)),
    ("welch_f64_odd_segments", "welch", "f64", 256 + 4 * 128 + 9, dict(nperseg=256)),
    ("csd_f64", "csd", "f64", 4000, dict(fs=2.0, nperseg=256)),
    ("csd_f64_pad_twosided", "csd", "f64", 3000,
     dict(nperseg=200, nfft=256, return_onesided=False)),
    ("csd_f32_promoted", "csd", "f32", 6000, dict(nperseg=512)),
    ("spectrogram_f64_psd", "spectrogram", "f64", 2000, dict(fs=8.0, nperseg=128)),
    ("spectrogram_f64_complex", "spectrogram", "f64", 2000,
     dict(nperseg=64, mode="complex")),
    ("spectrogram_f64_magnitude", "spectrogram", "f64", 3000,
     dict(nperseg=96, nfft=128, mode="magnitude")),
    ("spectrogram_f64_single_segment", "spectrogram", "f64", 256,
     dict(nperseg=256, mode="complex")),
    ("spectrogram_f64_single_segment_psd", "spectrogram", "f64", 300,
     dict(nperseg=256, mode="psd")),
    ("stft_f32", "stft", "f32", 3000, dict(fs=1e3, nperseg=128)),
    ("stft_f64_single_segment", "stft", "f64", 512, dict(nperseg=512)),
    ("stft_f64", "stft", "f64", 4000, dict(nperseg=256, noverlap=192)),
    ("coherence_f64", "coherence", "f64", 5000, dict(fs=2.0, nperseg=256)),
    ("coherence_f64_pad_hamming_none", "coherence", "f64", 4000,
     dict(nperseg=200, nfft=256, window="hamming", detrend="none")),
    ("coherence_f32_promoted", "coherence", "f32", 8192, dict(nperseg=512)),
    ("periodogram_f64", "periodogram", "f64", 3000, dict(fs=10.0)),
    ("periodogram_f64_hann_pad_spectrum", "periodogram", "f64", 2000,
     dict(window="hann", nfft=512, scaling="spectrum")),
    # istft: Zxx = the oracle's complex STFT of the case's signal (its
    # nperseg / noverlap in "stft"), inverted with the kwargs
    ("istft_defaults", "istft", "f64", 3000,
     dict(stft=dict(nperseg=128, noverlap=64))),
    ("istft_hamming_overlap", "istft", "f64", 4000,
     dict(stft=dict(nperseg=256, noverlap=192, window="hamming"),
          window="hamming", noverlap=192)),
    ("istft_padded", "istft", "f64", 2500,
     dict(stft=dict(nperseg=100, noverlap=50, nfft=128), nperseg=100,
          noverlap=50)),
    ("istft_two_sided_input", "istft", "f64", 1024,
     dict(stft=dict(nperseg=64, noverlap=32, twosided=True), nfft=64)),
]

ABI_PROBE = r"""
#include <stddef.h>
#include <stdio.h>
%s
int main(void) {
  printf("{\"InsightArray\": %%zu, \"C_DeviceInterface\": %%zu, "
         "\"CustomRuntimeParams\": %%zu, \"CustomRuntimeVersion\": %%zu, "
         "\"C_ProfilerEvent\": %%zu, "
         "\"off_numel\": %%zu, \"off_dtype\": %%zu, \"off_device_id\": %%zu, "
         "\"off_offset\": %%zu, \"off_ref_count\": %%zu, "
         "\"off_get_last_error\": %%zu, \"off_register_kernel\": %%zu}\n",
         sizeof(InsightArray), sizeof(C_DeviceInterface),
         sizeof(CustomRuntimeParams), sizeof(CustomRuntimeVersion),
         sizeof(C_ProfilerEvent),
         offsetof(InsightArray, numel), offsetof(InsightArray, dtype),
         offsetof(InsightArray, device_id), offsetof(InsightArray, offset),
         offsetof(InsightArray, ref_count),
         offsetof(C_DeviceInterface, get_last_error),
         offsetof(CustomRuntimeParams, register_kernel));
  return 0;
}
"""


def abi_layout(include_line: str, incdir: str, lang: str = "c++") -> dict:
    with tempfile.TemporaryDirectory() as d:
        src = os.path.join(d, "probe.cpp" if lang == "c++" else "probe.c")
        exe = os.path.join(d, "probe")
        with open(src, "w") as f:
            f.write(ABI_PROBE % include_line)
        cc = "/usr/bin/g++" if lang == "c++" else "/usr/bin/gcc"
        subprocess.run([cc, "-I" + incdir, src, "-o", exe], check=True)
        return json.loads(subprocess.run([exe], capture_output=True, text=True,
                                         check=True).stdout)


def signal(n, dtype, seed):
    rng = np.random.default_rng(seed)
    t = np.arange(n)
    x = (rng.standard_normal(n) + np.sin(2 * np.pi * 0.05 * t)
         + 0.5 * np.sin(2 * np.pi * 0.31 * t))
    return x.astype(np.float32 if dtype == "f32" else np.float64)


def main(ref_tree: str) -> None:
    out = {}
    for i, (name, op, dt, n, kw) in enumerate(CASES):
        x = signal(n, dt, 100 + i)
        out[name + "/x"] = x
        if op == "welch":
            # the reference throws on F32 welch/csd (item<double> on an F32
            # sum, spectral_analysis.cpp:63): record the promoted-F64 result
            f, p = ref_runner.welch(x.astype(np.float64), **kw)
            out[name + "/f"], out[name + "/Pxx"] = f, p
        elif op in ("csd", "coherence"):
            y = (0.7 * np.roll(x.astype(np.float64), 17)
                 + 0.3 * signal(n, "f64", 500 + i)).astype(x.dtype)
            out[name + "/y"] = y
            fn = ref_runner.csd if op == "csd" else ref_runner.coherence
            f, p = fn(x.astype(np.float64), y.astype(np.float64), **kw)
            out[name + "/f"], out[name + "/Pxx"] = f, p
        elif op == "istft":
            st = dict(kw["stft"])
            twosided = st.pop("twosided", False)
            _, _, z = so.stft(x.astype(np.float64), complex_output=True, **st)
            if twosided:  # the full spectrum, as a (nfft, n_frames) input
                step, S = so.framing(len(x), st["nperseg"], st["noverlap"], True)
                segs = so._segments(x.astype(np.float64), st["nperseg"], step, S)
                z = np.fft.fft(segs * so.get_window("hann", st["nperseg"])[None, :],
                               axis=1).T
            ik = {k: v for k, v in kw.items() if k != "stft"}
            out[name + "/Zxx"] = np.ascontiguousarray(z)
            out[name + "/out"] = ref_runner.istft(z, **ik)
        elif op == "periodogram":
            f, p = ref_runner.periodogram(x.astype(np.float64), **kw)
            out[name + "/f"], out[name + "/Pxx"] = f, p
        else:
            # F32 spectrogram/stft in the reference scatter an F32 column into
            # an F64 matrix without a cast (spectral_analysis.cpp:291-299 ->
            # scatter_reduce reads the F32 buffer as F64), so its F32 output is
            # not a spectrum: record the promoted-F64 result, as for welch.
            fn = ref_runner.stft if op == "stft" else ref_runner.spectrogram
            f, t, s = fn(x.astype(np.float64), **kw)
            out[name + "/f"], out[name + "/t"], out[name + "/Sxx"] = f, t, s
    np.savez_compressed(os.path.join(HERE, "reference_cases.npz"), **out)
    with open(os.path.join(HERE, "reference_cases.json"), "w") as f:
        json.dump([{"name": c[0], "op": c[1], "dtype": c[2], "n": c[3],
                    "kwargs": c[4]} for c in CASES], f, indent=1)
    lay = abi_layout('#include "insight/c_api/device_ext.h"\n'
                     '#include "insight/c_api/array.h"',
                     os.path.join(ref_tree, "include"))
    with open(os.path.join(HERE, "abi_layout.json"), "w") as f:
        json.dump(lay, f, indent=1)
    print("wrote", len(CASES), "cases and the ABI layout")


if __name__ == "__main__":
    if len(sys.argv) < 2:
        sys.exit("usage: make_golden.py <reference source tree>")
    main(sys.argv[1])
