"""ctypes binding of ``include/insight_b200.h``.

Loads ``libinsight_b200_backend.so`` from this package directory (built by
``insight_b200.build``) and describes the C ABI types.  Loading fails loudly:
there is no fallback implementation.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libinsight_b200_backend.so")

MAX_NDIM = 10

# InsightDType (include/insight/c_api/dtype.h)
DT_F32, DT_F64, DT_C32, DT_C64 = 9, 10, 11, 12
DEV_CPU, DEV_GPU = 0, 1
C_SUCCESS, C_FAILED, C_ERROR = 0, 2, 3

OP_WELCH, OP_CSD, OP_SPECTROGRAM, OP_STFT, OP_COHERENCE = 0, 1, 2, 3, 4


class InsightArray(ctypes.Structure):
    _fields_ = [
        ("data", ctypes.c_void_p),
        ("dims", ctypes.c_int64 * MAX_NDIM),
        ("strides", ctypes.c_int64 * MAX_NDIM),
        ("ndim", ctypes.c_int32),
        ("numel", ctypes.c_int64),
        ("dtype", ctypes.c_int32),
        ("device_type", ctypes.c_int32),
        ("device_id", ctypes.c_int32),
        ("offset", ctypes.c_int64),
        ("is_view", ctypes.c_int32),
        ("ref_count", ctypes.POINTER(ctypes.c_int32)),
    ]


KERNEL_FN = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.POINTER(ctypes.c_void_p),
                             ctypes.POINTER(ctypes.c_void_p))
REGISTER_FN = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_char_p, ctypes.c_int32,
                               ctypes.c_int32, ctypes.c_void_p)


class C_DeviceInterface(ctypes.Structure):
    # size + 53 function pointers + reserved[8]
    _fields_ = [("size", ctypes.c_size_t)] + [
        (n, ctypes.c_void_p) for n in (
            "initialize finalize init_device deinit_device set_device get_device "
            "synchronize_device get_device_count get_device_list "
            "device_memory_allocate device_memory_deallocate host_memory_allocate "
            "host_memory_deallocate memory_copy_h2d memory_copy_d2h memory_copy_d2d "
            "memory_copy_p2p device_memory_set device_memory_stats "
            "async_memory_copy_h2d async_memory_copy_d2h async_memory_copy_d2d "
            "async_memory_copy_p2p create_stream destroy_stream query_stream "
            "synchronize_stream stream_add_callback stream_wait_event create_event "
            "destroy_event record_event query_event synchronize_event elapsed_time "
            "get_compute_capability get_runtime_version get_driver_version "
            "get_multi_process get_max_threads_per_mp get_max_threads_per_block "
            "get_max_grid_dim_size get_device_name profiler_create profiler_destroy "
            "profiler_start profiler_stop profiler_reset profiler_begin_event "
            "profiler_end_event profiler_get_events get_last_error").split()
    ] + [("reserved", ctypes.c_void_p * 8)]


class CustomRuntimeVersion(ctypes.Structure):
    _fields_ = [("major", ctypes.c_size_t), ("minor", ctypes.c_size_t),
                ("patch", ctypes.c_size_t)]


class CustomRuntimeParams(ctypes.Structure):
    _fields_ = [
        ("size", ctypes.c_size_t),
        ("interface", ctypes.POINTER(C_DeviceInterface)),
        ("version", CustomRuntimeVersion),
        ("device_type", ctypes.c_char_p),
        ("sub_device_type", ctypes.c_char_p),
        ("register_kernel", REGISTER_FN),
        ("reserved", ctypes.c_char * 32),
    ]


class SpectralDesc(ctypes.Structure):
    _fields_ = [
        ("op", ctypes.c_int32),
        ("axis", ctypes.c_int32),
        ("fs", ctypes.c_double),
        ("window", ctypes.c_char_p),
        ("nperseg", ctypes.c_int64),
        ("noverlap", ctypes.c_int64),
        ("nfft", ctypes.c_int64),
        ("detrend", ctypes.c_char_p),
        ("return_onesided", ctypes.c_int32),
        ("scaling", ctypes.c_char_p),
        ("mode", ctypes.c_char_p),
        ("seg_begin", ctypes.c_int64),
        ("seg_end", ctypes.c_int64),
        ("raw_sums", ctypes.c_int32),
        ("avg_segments", ctypes.c_int64),
    ]


# Every symbol include/insight_b200.h declares.
EXPORTS = (
    "InitPluginGPU",
    "insight_b200_get_last_error",
    "insight_b200_welch_kernel",
    "insight_b200_csd_kernel",
    "insight_b200_spectrogram_kernel",
    "insight_b200_coherence_kernel",
    "insight_b200_istft_kernel",
    "insight_b200_welch",
    "insight_b200_csd",
    "insight_b200_spectrogram",
    "insight_b200_stft",
    "insight_b200_coherence",
    "insight_b200_periodogram",
    "insight_b200_istft_shape",
    "insight_b200_istft",
    "insight_b200_istft_async",
    "insight_b200_spectral_shape",
    "insight_b200_spectral",
    "insight_b200_finalize_sums",
    "insight_b200_launch_count",
    "insight_b200_welch_noalloc",
    "insight_b200_plan_create",
    "insight_b200_plan_execute",
    "insight_b200_plan_destroy",
)

_lib = None


def lib() -> ctypes.CDLL:
    """The loaded backend library (raises if it was not built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"{LIB_PATH} is missing: build it with `python -m insight_b200.build`")
        L = ctypes.CDLL(LIB_PATH)
        PA = ctypes.POINTER(InsightArray)
        L.insight_b200_get_last_error.restype = ctypes.c_char_p
        L.insight_b200_launch_count.restype = ctypes.c_int64
        L.InitPluginGPU.argtypes = [ctypes.POINTER(CustomRuntimeParams)]
        L.InitPluginGPU.restype = ctypes.c_int
        for n in ("insight_b200_welch_kernel", "insight_b200_csd_kernel",
                  "insight_b200_spectrogram_kernel", "insight_b200_coherence_kernel",
                  "insight_b200_istft_kernel"):
            f = getattr(L, n)
            f.argtypes = [ctypes.POINTER(ctypes.c_void_p), ctypes.POINTER(ctypes.c_void_p)]
            f.restype = ctypes.c_int
        L.insight_b200_welch.argtypes = [
            PA, ctypes.c_double, ctypes.c_char_p, ctypes.c_int64, ctypes.c_int64,
            ctypes.c_int64, ctypes.c_char_p, ctypes.c_int, ctypes.c_char_p, PA, PA]
        L.insight_b200_csd.argtypes = [
            PA, PA, ctypes.c_double, ctypes.c_char_p, ctypes.c_int64, ctypes.c_int64,
            ctypes.c_int64, ctypes.c_char_p, ctypes.c_int, ctypes.c_char_p, PA, PA]
        L.insight_b200_spectrogram.argtypes = [
            PA, ctypes.c_double, ctypes.c_char_p, ctypes.c_int64, ctypes.c_int64,
            ctypes.c_int64, ctypes.c_char_p, ctypes.c_int, ctypes.c_char_p, PA, PA, PA]
        L.insight_b200_stft.argtypes = [
            PA, ctypes.c_double, ctypes.c_char_p, ctypes.c_int64, ctypes.c_int64,
            ctypes.c_int64, PA, PA, PA]
        L.insight_b200_coherence.argtypes = [
            PA, PA, ctypes.c_double, ctypes.c_char_p, ctypes.c_int64, ctypes.c_int64,
            ctypes.c_int64, ctypes.c_char_p, PA, PA]
        L.insight_b200_periodogram.argtypes = [
            PA, ctypes.c_double, ctypes.c_char_p, ctypes.c_int64, ctypes.c_char_p,
            ctypes.c_int, ctypes.c_char_p, PA, PA]
        L.insight_b200_istft_shape.argtypes = [
            PA, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
            ctypes.POINTER(ctypes.c_int64), ctypes.POINTER(ctypes.c_int64)]
        L.insight_b200_istft.argtypes = [
            PA, ctypes.c_double, ctypes.c_char_p, ctypes.c_int64, ctypes.c_int64,
            ctypes.c_int64, PA]
        L.insight_b200_istft_async.argtypes = [
            PA, ctypes.c_char_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, PA,
            ctypes.c_void_p, ctypes.c_int]
        L.insight_b200_istft_async.restype = ctypes.c_int
        PD = ctypes.POINTER(SpectralDesc)
        PI64 = ctypes.POINTER(ctypes.c_int64)
        L.insight_b200_spectral_shape.argtypes = [PD, PA, PI64, PI64, PI64]
        L.insight_b200_spectral.argtypes = [PD, PA, PA, PA, PA, PA, ctypes.c_void_p,
                                            ctypes.c_int]
        L.insight_b200_finalize_sums.argtypes = [PD, ctypes.c_int64, ctypes.c_int32,
                                                 PA, ctypes.c_void_p]
        L.insight_b200_welch_noalloc.argtypes = [
            ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_int64,
            ctypes.c_int64, ctypes.c_int64, ctypes.c_double, ctypes.c_char_p,
            ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_char_p,
            ctypes.c_int32, ctypes.c_char_p, ctypes.c_void_p, ctypes.c_void_p]
        L.insight_b200_welch_noalloc.restype = ctypes.c_int
        L.insight_b200_plan_create.argtypes = [PD, PA, PA, PA, ctypes.c_void_p,
                                               ctypes.POINTER(ctypes.c_void_p)]
        L.insight_b200_plan_execute.argtypes = [ctypes.c_void_p, ctypes.c_void_p,
                                                ctypes.c_int]
        L.insight_b200_plan_destroy.argtypes = [ctypes.c_void_p]
        for n in ("insight_b200_plan_create", "insight_b200_plan_execute",
                  "insight_b200_plan_destroy"):
            getattr(L, n).restype = ctypes.c_int
        for n in ("insight_b200_welch", "insight_b200_csd", "insight_b200_spectrogram",
                  "insight_b200_stft", "insight_b200_coherence",
                  "insight_b200_periodogram", "insight_b200_istft_shape",
                  "insight_b200_istft", "insight_b200_spectral_shape",
                  "insight_b200_spectral", "insight_b200_finalize_sums"):
            getattr(L, n).restype = ctypes.c_int
        _lib = L
    return _lib


def last_error() -> str:
    return (lib().insight_b200_get_last_error() or b"").decode()


def check(status: int, what: str) -> None:
    if status != C_SUCCESS:
        raise RuntimeError(f"{what}: {last_error()}")


def launch_count() -> int:
    return int(lib().insight_b200_launch_count())


# ---------------------------------------------------------------------------
# InsightArray descriptors for numpy arrays (host) and torch tensors (device).
# ---------------------------------------------------------------------------
_NP_DT = {"float32": DT_F32, "float64": DT_F64, "complex64": DT_C32,
          "complex128": DT_C64}


def _fill(a: InsightArray, ptr: int, shape, strides, dtype: int, dev_type: int,
          dev_id: int, offset: int = 0) -> InsightArray:
    nd = len(shape)
    if nd > MAX_NDIM:
        raise ValueError(f"InsightArray holds at most {MAX_NDIM} dimensions")
    a.data = ptr
    a.ndim = nd
    a.dims[:nd] = shape
    a.strides[:nd] = strides
    n = 1
    for d in shape:
        n *= d
    a.numel = n
    a.dtype = dtype
    a.device_type = dev_type
    a.device_id = dev_id
    a.offset = offset
    return a


def from_numpy(x) -> InsightArray:
    """Descriptor of a numpy array (CPU).  Strides are converted to elements."""
    dt = _NP_DT[str(x.dtype)]
    item = x.dtype.itemsize
    strides = [s // item for s in x.strides]
    return _fill(InsightArray(), x.ctypes.data, tuple(x.shape), strides, dt,
                 DEV_CPU, 0)


_TORCH_DT = {"torch.float32": DT_F32, "torch.float64": DT_F64,
             "torch.complex64": DT_C32, "torch.complex128": DT_C64}


def from_torch(t) -> InsightArray:
    """Descriptor of a torch tensor (CUDA or CPU), strides/offset in elements."""
    dt = _TORCH_DT[str(t.dtype)]
    if t.is_cuda:
        dev_type, dev_id = DEV_GPU, t.device.index
    else:
        dev_type, dev_id = DEV_CPU, 0
    base = t.untyped_storage().data_ptr()
    return _fill(InsightArray(), base, t.shape, t.stride(), dt, dev_type, dev_id,
                 t.storage_offset())


def as_array(x) -> InsightArray:
    if x is None:
        return None
    if hasattr(x, "untyped_storage"):
        return from_torch(x)
    return from_numpy(x)


def ptr(a):
    return ctypes.byref(a) if a is not None else None
