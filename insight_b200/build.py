"""Build libinsight_b200_backend.so in-tree (sm_100a).

    python -m insight_b200.build          # or insight_b200.build.build()

CUDA sources are compiled by nvcc for ``sm_100a`` only; host C++ sources by
the host compiler with the CUDA include path; everything is linked into
``insight_b200/libinsight_b200_backend.so`` next to this file, so the shared
object travels with the source tree.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libinsight_b200_backend.so")

CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA_HOME, "bin", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CU_SOURCES = ["spectral_f32.cu", "spectral_f64.cu", "spectral_util.cu",
              "spectral_noalloc.cu", "spectral_istft.cu"]
CPP_SOURCES = ["launch.cpp", "frontend.cpp", "plugin.cpp", "windows.cpp"]
HEADERS = ["fft_core.cuh", "spectral_kernels.cuh", "spectral_dispatch.cuh",
           "spectral_accum_fast.cuh", "spectral_istft.cuh", "spectral_stft_ws.cuh",
           "spectral_stft_tma.cuh",
           "launch.h", "frontend.h", "windows.h"]


def _host_cxx() -> str:
    for c in ("/usr/bin/g++", shutil.which("g++") or ""):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("no host C++ compiler found")


def _newer(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return False
    t = os.path.getmtime(target)
    return all(os.path.getmtime(d) <= t for d in deps)


def _compile(cmd: list[str]) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("compile failed:\n" + " ".join(cmd) + "\n" + r.stdout + r.stderr)


def build(verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    inc = ["-I" + CSRC, "-I" + os.path.join(ROOT, "include"),
           "-I" + os.path.join(CUDA_HOME, "include")]
    hdrs = [os.path.join(CSRC, h) for h in HEADERS] + [
        os.path.join(ROOT, "include", "insight_b200.h")]
    jobs, objs = [], []
    for s in CU_SOURCES:
        src = os.path.join(CSRC, s)
        obj = os.path.join(BUILD, s + ".o")
        objs.append(obj)
        if not _newer(obj, [src] + hdrs):
            jobs.append([NVCC, "-std=c++17", *ARCH, "-O3", "-lineinfo",
                         "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
                         *inc, "-c", src, "-o", obj])
    cxx = _host_cxx()
    for s in CPP_SOURCES:
        src = os.path.join(CSRC, s)
        obj = os.path.join(BUILD, s + ".o")
        objs.append(obj)
        if not _newer(obj, [src] + hdrs):
            jobs.append([cxx, "-std=c++17", "-O2", "-fPIC", "-fvisibility=hidden",
                         "-Wall", *inc, "-c", src, "-o", obj])
    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(8, len(jobs))) as ex:
            for f in [ex.submit(_compile, j) for j in jobs]:
                f.result()
    if jobs or not os.path.exists(LIB):
        cmd = [NVCC, *ARCH, "-shared", "-o", LIB, *objs,
               "-L" + os.path.join(CUDA_HOME, "lib64"), "-lcudart"]
        _compile(cmd)
    if verbose:
        print("built", LIB)
    return LIB


if __name__ == "__main__":
    build(verbose=True)
    sys.exit(0)
