"""Reference outputs at the benchmark configurations' own parameters.

Runs the reference's own ins::signal::welch / csd / stft, compiled from its
sources into oracle/_ref (``make -C oracle ref REF_DIR=<reference tree>``), on
one channel (or pair) of each configuration's seeded input
(tests/golden/config_inputs.py) and writes the outputs to
tests/golden/reference_configs.npz.  The inputs are not stored: the tests
regenerate them from the same seeds.

    python tests/golden/make_config_golden.py

The reference throws on F32 welch / csd (spectral_analysis.cpp:63 takes
item<double> of an F32 sum) and reads an F32 stft column as F64 in its
scatter, so f32 inputs are given to it promoted to F64, as in
make_golden.py; the B200 path computes in f32 and is held to 1e-5 of the
largest bin of these outputs.
"""
from __future__ import annotations

import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, HERE)

from oracle import ref_runner  # noqa: E402
import config_inputs as ci  # noqa: E402


def main() -> None:
    ref_runner.set_threads(os.cpu_count() or 1)
    out = {}
    for name, make, op, kw in ci.CASES:
        t0 = time.perf_counter()
        if op == "csd":
            x, y = make()
            f, p = ref_runner.csd(x.astype(np.float64), y.astype(np.float64), **kw)
            out[name + "/f"], out[name + "/Pxx"] = f, p
        elif op == "welch":
            x = make()
            f, p = ref_runner.welch(x.astype(np.float64), **kw)
            out[name + "/f"], out[name + "/Pxx"] = f, p
        else:
            x = make()
            f, t, s = ref_runner.stft(x.astype(np.float64), **kw)
            out[name + "/f"], out[name + "/t"], out[name + "/Sxx"] = f, t, s
        print(f"{name}: {time.perf_counter() - t0:.1f} s", flush=True)
    np.savez_compressed(os.path.join(HERE, "reference_configs.npz"), **out)
    print("wrote", len(ci.CASES), "configuration cases")


if __name__ == "__main__":
    main()
