"""The stream, event-timing and compile-log entry points of the C ABI,
called through ctypes as a binding other than the bundled one would."""

from __future__ import annotations

import ctypes

import pytest

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def lib(mx):
    from phew_b200 import _native

    return _native.load()


def test_stream_and_event_timing(lib, mx):
    import torch

    from phew_b200 import _native

    st, e0, e1 = ctypes.c_void_p(), ctypes.c_void_p(), ctypes.c_void_p()
    assert lib.phew_stream_create(ctypes.byref(st)) == 0 and st.value
    assert lib.phew_event_create(ctypes.byref(e0)) == 0
    assert lib.phew_event_create(ctypes.byref(e1)) == 0
    buf = torch.empty(512 * 1024 * 1024, dtype=torch.uint8, device="cuda")  # 512 MB write
    assert lib.phew_event_record(e0, st) == 0
    assert lib.phew_l2_flush(ctypes.c_void_p(buf.data_ptr()), ctypes.c_size_t(buf.numel()), st) == 0
    assert lib.phew_event_record(e1, st) == 0
    ms = ctypes.c_float()
    assert lib.phew_event_elapsed_ms(e0, e1, ctypes.byref(ms)) == 0
    # 512 MB written: between 10 us and 100 ms on any B200 clock
    assert 0.01 < ms.value < 100.0, ms.value
    for e in (e0, e1):
        assert lib.phew_event_destroy(e) == 0
    assert lib.phew_stream_destroy(st) == 0
    assert lib.phew_event_elapsed_ms(None, None, ctypes.byref(ms)) == _native.PHEW_ERR_INVALID


def test_compile_log(lib, mx):
    from phew_b200 import _native

    h = ctypes.c_uint64()
    bad = b'extern "C" __global__ void broken_kernel(float* p) { p[0] = undefined_name; }'
    assert lib.phew_compile(bad, b"broken_kernel", ctypes.byref(h)) == _native.PHEW_ERR_COMPILE
    n = lib.phew_compile_log(None, 0)
    buf = ctypes.create_string_buffer(n + 1)
    assert lib.phew_compile_log(buf, n + 1) == n
    assert b"undefined_name" in buf.value
    good = b'extern "C" __global__ void fine_kernel(float* p) { p[threadIdx.x] = 1.0f; }'
    assert lib.phew_compile(good, b"fine_kernel", ctypes.byref(h)) == 0
    n2 = lib.phew_compile_log(None, 0)
    buf2 = ctypes.create_string_buffer(n2 + 1)
    lib.phew_compile_log(buf2, n2 + 1)
    assert b"undefined_name" not in buf2.value  # the clean compile replaced the log
