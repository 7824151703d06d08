"""ctypes binding of ``libphew_b200.so`` (declared in ``include/phew_b200.h``).

The library is the only way this package reaches the GPU: there is no
Python or CPU fallback.  Loading fails loudly when the library is missing.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libphew_b200.so"

PHEW_OK = 0
PHEW_ERR_INVALID = 1
PHEW_ERR_CUDA = 2
PHEW_ERR_COMPILE = 3
PHEW_ERR_UNSUPPORTED = 4
PHEW_ERR_TIMEOUT = 5
PHEW_ERR_NOT_FOUND = 6

PHEW_F32 = 0
PHEW_F16 = 1
PHEW_BF16 = 2

REDUCE_OPS = {"sum": 0, "mean": 1, "max": 2, "min": 3, "prod": 4}

# Every symbol the header declares; tests check that each one is exported.
EXPORTED_SYMBOLS = (
    "phew_abi_version",
    "phew_last_error",
    "phew_init",
    "phew_device_query",
    "phew_compile",
    "phew_launch",
    "phew_launch_count",
    "phew_compile_cache_size",
    "phew_compile_log",
    "phew_stream_create",
    "phew_stream_destroy",
    "phew_event_create",
    "phew_event_record",
    "phew_event_elapsed_ms",
    "phew_event_destroy",
    "phew_test_inject_stall",
    "phew_rms_norm",
    "phew_layer_norm",
    "phew_rope",
    "phew_softmax",
    "phew_reduce_var",
    "phew_dequantize",
    "phew_quantize",
    "phew_copy_strided_to",
    "phew_reduce",
    "phew_copy_strided",
    "phew_l2_flush",
    "phew_gemm",
    "phew_gemm_batched2",
    "phew_sdpa_supported",
    "phew_sdpa",
    "phew_sdpa_strided",
    "phew_fill",
    "phew_fill_host",
    "phew_compare_scratch_bytes",
    "phew_compare",
    "phew_compare_static",
)


class PhewError(RuntimeError):
    """A native call returned a non-zero status."""

    def __init__(self, status: int, message: str) -> None:
        super().__init__(f"[phew status {status}] {message}")
        self.status = status


class PhewCompileError(PhewError):
    """NVRTC rejected an emitted or user-supplied kernel source."""


class DeviceInfo(ctypes.Structure):
    _fields_ = [
        ("sm_count", ctypes.c_int),
        ("cc_major", ctypes.c_int),
        ("cc_minor", ctypes.c_int),
        ("max_smem_per_block_optin", ctypes.c_int),
        ("l2_bytes", ctypes.c_int64),
        ("hbm_bytes", ctypes.c_int64),
        ("name", ctypes.c_char * 128),
    ]


class CompareStats(ctypes.Structure):
    _fields_ = [
        ("sum_abs_base", ctypes.c_double),
        ("mean_abs_base", ctypes.c_double),
        ("max_abs_diff", ctypes.c_double),
        ("atol_used", ctypes.c_double),
        ("rtol_used", ctypes.c_double),
        ("n", ctypes.c_int64),
        ("n_nonfinite_base", ctypes.c_int64),
        ("n_mismatch", ctypes.c_int64),
        ("n_nan_any", ctypes.c_int64),
        ("skipped", ctypes.c_int32),
        ("passed", ctypes.c_int32),
    ]


_lib = None
_lock = threading.Lock()

_vp = ctypes.c_void_p
_i64 = ctypes.c_int64
_int = ctypes.c_int

_SIGNATURES = {
    "phew_abi_version": ([], _int),
    "phew_last_error": ([ctypes.c_char_p, ctypes.c_size_t], _int),
    "phew_init": ([_int], _int),
    "phew_device_query": ([_int, ctypes.POINTER(DeviceInfo)], _int),
    "phew_compile": ([ctypes.c_char_p, ctypes.c_char_p, ctypes.POINTER(ctypes.c_uint64)], _int),
    "phew_compile_log": ([ctypes.c_char_p, ctypes.c_size_t], _int),
    "phew_stream_create": ([ctypes.POINTER(ctypes.c_void_p)], _int),
    "phew_stream_destroy": ([ctypes.c_void_p], _int),
    "phew_event_create": ([ctypes.POINTER(ctypes.c_void_p)], _int),
    "phew_event_record": ([ctypes.c_void_p, ctypes.c_void_p], _int),
    "phew_event_elapsed_ms": ([ctypes.c_void_p, ctypes.c_void_p, ctypes.POINTER(ctypes.c_float)], _int),
    "phew_event_destroy": ([ctypes.c_void_p], _int),
    "phew_launch": (
        [ctypes.c_uint64, ctypes.POINTER(ctypes.c_void_p), _int]
        + [ctypes.c_uint] * 6
        + [ctypes.c_size_t, _vp],
        _int,
    ),
    "phew_launch_count": ([ctypes.POINTER(ctypes.c_uint64)], _int),
    "phew_compile_cache_size": ([], _int),
    "phew_rms_norm": ([_vp, _vp, _vp, _i64, _i64, ctypes.c_float, _int, _vp], _int),
    "phew_layer_norm": ([_vp, _vp, _vp, _vp, _i64, _i64, ctypes.c_float, _int, _vp], _int),
    "phew_rope": (
        [_vp, _vp, _i64, _i64, _i64, _int, _int, ctypes.c_float, ctypes.c_float, _i64, _int, _vp],
        _int,
    ),
    "phew_softmax": ([_vp, _vp, _i64, _i64, _int, _vp], _int),
    "phew_reduce_var": ([_vp, _vp, _i64, _i64, _i64, _int, _int, _vp], _int),
    "phew_dequantize": ([_vp, _vp, _vp, _vp, _i64, _i64, _int, _int, _int, _vp], _int),
    "phew_copy_strided_to": (
        [_vp, _vp, _int, ctypes.POINTER(_i64), ctypes.POINTER(_i64), ctypes.POINTER(_i64), _int, _vp],
        _int,
    ),
    "phew_reduce": ([_int, _vp, _vp, _i64, _i64, _i64, _int, _vp], _int),
    "phew_copy_strided": (
        [_vp, _vp, _int, ctypes.POINTER(_i64), ctypes.POINTER(_i64), _int, _vp],
        _int,
    ),
    "phew_l2_flush": ([_vp, ctypes.c_size_t, _vp], _int),
    "phew_gemm": (
        [_vp, _vp, _vp] + [_i64] * 10 + [_int, _int, _int, _int, ctypes.c_float, _vp, _vp],
        _int,
    ),
    "phew_gemm_batched2": (
        [_vp, _vp, _vp] + [_i64] * 13 + [_int, _int, _int, _vp, _vp],
        _int,
    ),
    "phew_sdpa_supported": ([_i64, _i64, _int], _int),
    "phew_sdpa": (
        [_vp, _vp, _vp, _vp, _i64, _i64, _i64, ctypes.c_float, _int, _int, _vp, _vp],
        _int,
    ),
    "phew_sdpa_strided": (
        [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, ctypes.POINTER(_i64), ctypes.POINTER(_i64),
         ctypes.POINTER(_i64), ctypes.c_float, _int, _int, _vp, _vp],
        _int,
    ),
    "phew_fill": (
        [_vp, _i64, _i64, _int, _int, ctypes.c_uint64, ctypes.c_uint64, ctypes.c_float, _vp],
        _int,
    ),
    "phew_compare_scratch_bytes": ([_i64], ctypes.c_size_t),
    "phew_compare": (
        [_vp, _vp, _i64, _int, ctypes.c_double, ctypes.c_double, _vp, ctypes.c_size_t, _vp, _vp],
        _int,
    ),
    "phew_compare_static": (
        [_vp, _vp, _i64, _int, ctypes.c_double, ctypes.c_double, _vp, _vp],
        _int,
    ),
}


def load(path: str | os.PathLike | None = None) -> ctypes.CDLL:
    """Load (once) and return the native library.  Raises if it is missing."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        p = Path(path) if path else LIB_PATH
        if not p.exists():
            raise ImportError(
                f"phew_b200 native library not found at {p}; build it with "
                "`python -m phew_b200.build` (there is no CPU fallback)"
            )
        lib = ctypes.CDLL(str(p))
        for name, (argtypes, restype) in _SIGNATURES.items():
            fn = getattr(lib, name)
            fn.argtypes = argtypes
            fn.restype = restype
        _lib = lib
        return lib


def last_error() -> str:
    lib = load()
    buf = ctypes.create_string_buffer(8192)
    lib.phew_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(status: int, what: str = "") -> None:
    """Raise PhewError (or PhewCompileError) for a non-zero status."""
    if status == PHEW_OK:
        return
    msg = last_error()
    if what:
        msg = f"{what}: {msg}"
    if status == PHEW_ERR_COMPILE:
        raise PhewCompileError(status, msg)
    raise PhewError(status, msg)


def call(name: str, *args):
    """Call a status-returning entry point and raise on failure."""
    lib = load()
    check(getattr(lib, name)(*args), name)


def launch_count() -> int:
    """Kernels the native library has launched in this process (graph
    captures count the launches they record)."""
    n = ctypes.c_uint64(0)
    call("phew_launch_count", ctypes.byref(n))
    return int(n.value)
