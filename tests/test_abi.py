"""C ABI of libinsight_b200_backend.so, checked without a GPU.

* the library loads and exports every symbol include/insight_b200.h declares;
* the ABI types have the reference's layout (tests/golden/abi_layout.json was
  measured on the reference's own include/insight/c_api headers);
* argument validation mirrors the reference's messages and happens before any
  device call, and the plugin factory rejects mismatched struct sizes.
"""
import ctypes
import json
import os
import re
import subprocess
import tempfile

import numpy as np
import pytest

from insight_b200 import _abi

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "insight_b200.h")


def declared_symbols():
    src = open(HEADER).read()
    return sorted(set(re.findall(r"INSIGHT_B200_API\s+[\w\s\*]+?\b(\w+)\s*\(", src)))


def test_header_declares_what_the_binding_lists():
    assert declared_symbols() == sorted(_abi.EXPORTS)


def test_library_exports_every_declared_symbol():
    lib = _abi.lib()
    for name in declared_symbols():
        assert hasattr(lib, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", _abi.LIB_PATH],
                         capture_output=True, text=True, check=True).stdout
    exported = {l.split()[-1] for l in out.splitlines() if " T " in l}
    assert set(declared_symbols()) <= exported


@pytest.mark.parametrize("lang", ["c", "c++"])
def test_abi_layout_matches_reference(lang):
    from tests.golden.make_golden import abi_layout
    expect = json.load(open(os.path.join(ROOT, "tests", "golden", "abi_layout.json")))
    got = abi_layout('#include "insight_b200.h"', os.path.join(ROOT, "include"), lang)
    assert got == expect


def test_ctypes_mirror_layout():
    expect = json.load(open(os.path.join(ROOT, "tests", "golden", "abi_layout.json")))
    assert ctypes.sizeof(_abi.InsightArray) == expect["InsightArray"]
    assert ctypes.sizeof(_abi.C_DeviceInterface) == expect["C_DeviceInterface"]
    assert ctypes.sizeof(_abi.CustomRuntimeParams) == expect["CustomRuntimeParams"]
    assert _abi.InsightArray.offset.offset == expect["off_offset"]
    assert _abi.C_DeviceInterface.get_last_error.offset == expect["off_get_last_error"]
    assert (_abi.CustomRuntimeParams.register_kernel.offset
            == expect["off_register_kernel"])


def test_plugin_rejects_size_mismatch():
    lib = _abi.lib()
    iface = _abi.C_DeviceInterface()
    iface.size = ctypes.sizeof(_abi.C_DeviceInterface) - 8
    params = _abi.CustomRuntimeParams()
    params.size = ctypes.sizeof(_abi.CustomRuntimeParams)
    params.interface = ctypes.pointer(iface)
    assert lib.InitPluginGPU(ctypes.byref(params)) == _abi.C_ERROR
    iface.size = ctypes.sizeof(_abi.C_DeviceInterface)
    params.size = 8
    assert lib.InitPluginGPU(ctypes.byref(params)) == _abi.C_ERROR


def _no_gpu():
    try:
        import torch
        return not torch.cuda.is_available()
    except Exception:
        return True


@pytest.mark.skipif(not _no_gpu(), reason="checks the no-device path")
def test_plugin_fails_loudly_without_a_gpu():
    lib = _abi.lib()
    iface = _abi.C_DeviceInterface()
    iface.size = ctypes.sizeof(_abi.C_DeviceInterface)
    params = _abi.CustomRuntimeParams()
    params.size = ctypes.sizeof(_abi.CustomRuntimeParams)
    params.interface = ctypes.pointer(iface)
    assert lib.InitPluginGPU(ctypes.byref(params)) == _abi.C_FAILED
    assert _abi.last_error()


def _welch(x, **kw):
    lib = _abi.lib()
    xa = _abi.from_numpy(x)
    out = np.zeros(4096)
    oa = _abi.from_numpy(out[: kw.get("F", 129)])
    return lib.insight_b200_welch(
        ctypes.byref(xa), 1.0, kw.get("window", "hann").encode(), kw.get("nperseg", 256),
        kw.get("noverlap", 0), kw.get("nfft", 0), b"constant", 1, b"density", None,
        ctypes.byref(oa))


@pytest.mark.parametrize("kw,msg", [
    (dict(n=100, nperseg=256), "csd: signal too short for given nperseg"),
    (dict(n=1000, nperseg=0), "nperseg must be positive"),
    (dict(n=1000, nperseg=256, noverlap=256), "noverlap must be less than nperseg"),
    (dict(n=1000, nperseg=100), "nfft must be a power of two"),
    (dict(n=1000, nperseg=256, nfft=128), "nfft must be >= nperseg"),
    (dict(n=1000, nperseg=128, window="nope"), "get_window: unknown window name 'nope'"),
])
def test_validation_messages(kw, msg):
    x = np.zeros(kw.pop("n"))
    assert _welch(x, **kw) == _abi.C_FAILED
    assert msg in _abi.last_error()


def test_dtype_is_checked():
    lib = _abi.lib()
    x = np.zeros(1000, dtype=np.complex64)
    xa = _abi.from_numpy(x)
    out = np.zeros(129)
    assert lib.insight_b200_welch(ctypes.byref(xa), 1.0, b"hann", 256, 0, 0,
                                  b"constant", 1, b"density", None,
                                  ctypes.byref(_abi.from_numpy(out))) == _abi.C_FAILED
    assert "F32 or F64" in _abi.last_error()


def test_shape_query():
    lib = _abi.lib()
    d = _abi.SpectralDesc()
    d.op = _abi.OP_STFT
    d.axis = 0
    d.nperseg = 2048
    d.noverlap = 1536
    d.return_onesided = 1
    x = np.zeros((1 << 14, 3), dtype=np.float32)
    c, s, f = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int64()
    assert lib.insight_b200_spectral_shape(ctypes.byref(d), ctypes.byref(
        _abi.from_numpy(x)), ctypes.byref(c), ctypes.byref(s), ctypes.byref(f)) == 0
    assert (c.value, s.value, f.value) == (3, ((1 << 14) - 2048) // 512 + 1, 1025)
