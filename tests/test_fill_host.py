"""The host twin of the sweep's input generator (``phew_fill_host``): the
same counter-based draws as the device's ``phew_fill``, restated here in
numpy, independent of the thread count, with round-to-nearest-even 16-bit
storage.  CPU only (the function touches no device)."""

from __future__ import annotations

import ctypes

import ml_dtypes
import numpy as np
import pytest

BF16 = np.dtype(ml_dtypes.bfloat16)
M64 = (1 << 64) - 1


@pytest.fixture(scope="module")
def lib():
    from phew_b200 import _native
    from phew_b200.build import build

    build()
    return _native.load()


def _mix64(z: int) -> int:
    z = (z + 0x9E3779B97F4A7C15) & M64
    z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & M64
    z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & M64
    return z ^ (z >> 31)


def _draw(seed: int, stream: int, i: int) -> int:
    return _mix64(_mix64(_mix64(seed) ^ stream) ^ i)


def _u24(bits: int) -> float:
    return ((bits & 0xFFFFFF) + 1.0) / 16777216.0


def _fill(lib, n, cols, dtype, kind, seed, stream, scale, threads=0):
    np_t = {0: np.float32, 1: np.float16, 2: np.uint16}[dtype]
    out = np.empty(n, np_t)
    st = lib.phew_fill_host(ctypes.c_void_p(out.ctypes.data), ctypes.c_int64(n), ctypes.c_int64(cols),
                            dtype, kind, ctypes.c_uint64(seed), ctypes.c_uint64(stream),
                            ctypes.c_float(scale), threads)
    assert st == 0
    return out.view(BF16) if dtype == 2 else out


def test_normal_draws_follow_the_generator(lib):
    seed, stream = 11, 0x1234_5678_9ABC
    got = _fill(lib, 4097, 64, 0, 0, seed, stream, 0.5)
    # Box-Muller pairs: elements 2k and 2k + 1 share draw k
    for i in (0, 1, 7, 1000, 4095, 4096):
        b = _draw(seed, stream, i // 2)
        trig = np.cos if i % 2 == 0 else np.sin
        want = np.sqrt(-2.0 * np.log(_u24(b))) * trig(2 * np.pi * _u24(b >> 32)) * 0.5
        assert abs(float(got[i]) - want) <= 2e-6 * max(1.0, abs(want)), (i, got[i], want)


def _mix64_np(z):
    z = z + np.uint64(0x9E3779B97F4A7C15)
    z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
    z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
    return z ^ (z >> np.uint64(31))


@pytest.mark.parametrize("dtype", [0, 2])
def test_normal_draws_accuracy(lib, dtype):
    """Every element of a 2^20 sample against the transform in float64: the
    host's series forms of ln and cos / sin (vectorised) stay within a few
    fp32 ulps (and 16-bit values within one rounding of the exact value)."""
    n, seed, stream, scale = (1 << 20) + 1, 21, 0xABCDEF, 1.5
    got = _fill(lib, n, 4096, dtype, 0, seed, stream, scale).astype(np.float64)
    k = np.arange((n + 1) // 2, dtype=np.uint64)
    with np.errstate(over="ignore"):
        base = _mix64_np(_mix64_np(np.uint64(seed)) ^ np.uint64(stream))
        b = _mix64_np(base ^ k)
    u1 = ((b & np.uint64(0xFFFFFF)).astype(np.float64) + 1.0) / 16777216.0
    u2 = (((b >> np.uint64(32)) & np.uint64(0xFFFFFF)).astype(np.float64) + 1.0) / 16777216.0
    r = np.sqrt(-2.0 * np.log(u1)) * scale
    want = np.empty(2 * len(k))
    want[0::2] = r * np.cos(2 * np.pi * u2)
    want[1::2] = r * np.sin(2 * np.pi * u2)
    want = want[:n]
    tol = 2e-6 if dtype == 0 else 2.0 ** -8
    err = np.abs(got - want) / np.maximum(1.0, np.abs(want))
    assert err.max() <= tol, (err.max(), int(err.argmax()))


def test_thread_count_does_not_change_values(lib):
    n = 3 * (1 << 20) + 5  # odd: the last pair has one element
    a = _fill(lib, n, 4096, 2, 0, 3, 99, 1.0, threads=1)
    b = _fill(lib, n, 4096, 2, 0, 3, 99, 1.0, threads=7)
    assert np.array_equal(a.view(np.uint16), b.view(np.uint16))
    f = a.astype(np.float32)
    assert abs(f.mean()) < 5e-3 and abs(f.std() - 1) < 5e-3


def test_one_hot_rows_and_constant(lib):
    rows, cols = 33, 257
    a = _fill(lib, rows * cols, cols, 2, 2, 5, 17, 1.0).astype(np.float32).reshape(rows, cols)
    assert np.all(a.sum(-1) == 1.0) and np.all((a == 0) | (a == 1))
    for r in (0, 32):
        assert a[r, _draw(5, 17, r) % cols] == 1.0
    c = _fill(lib, 100, 10, 1, 3, 0, 0, 0.75)
    assert np.all(c == np.float16(0.75))


@pytest.mark.parametrize("dtype", [1, 2])
def test_sixteen_bit_rounding_matches_numpy(lib, dtype):
    vals = np.array([0.0, -0.0, 1e-8, 2.98e-8, 2.99e-8, 5.96e-8, 9e-8, 6.0976e-5, 6.104e-5,
                     0.33333334, 1.0 + 2 ** -9, 1.0 + 3 * 2 ** -9, 65504, 65519, 65520, 1e6,
                     -1e-7, 1e-39, -3e38, np.inf, -np.inf, np.nan], np.float32)
    want = vals.astype(np.float16 if dtype == 1 else BF16).view(np.uint16)
    got = np.array([_fill(lib, 1, 1, dtype, 3, 0, 0, float(v)).view(np.uint16)[0] for v in vals])
    nan = np.isnan(vals)
    assert np.array_equal(got[~nan], want[~nan])
    # NaN stays NaN (quiet)
    g = got[nan][0]
    assert (g & (0x7C00 if dtype == 1 else 0x7F80)) == (0x7C00 if dtype == 1 else 0x7F80) and g & 0x3FF


def test_rejects_bad_arguments(lib):
    from phew_b200 import _native

    assert lib.phew_fill_host(None, ctypes.c_int64(4), ctypes.c_int64(4), 0, 0, ctypes.c_uint64(0),
                              ctypes.c_uint64(0), ctypes.c_float(1.0), 1) == _native.PHEW_ERR_INVALID
    buf = np.empty(4, np.float32)
    assert lib.phew_fill_host(ctypes.c_void_p(buf.ctypes.data), ctypes.c_int64(4), ctypes.c_int64(4), 9, 0,
                              ctypes.c_uint64(0), ctypes.c_uint64(0), ctypes.c_float(1.0), 1) == _native.PHEW_ERR_INVALID


def test_bf16_subnormal_draws(lib):
    """Normals scaled to bf16 subnormals (the sweep's subnormal variant) take
    the double-precision path; they match rounding the fp32 draws scaled in
    double, except where the order of the two roundings decides a tie."""
    n = 1 << 20
    f = _fill(lib, n, 4096, 0, 0, 5, 9, 1.0).astype(np.float64)
    got = _fill(lib, n, 4096, 2, 0, 5, 9, 1e-39).view(np.uint16)
    want = (f * np.float64(np.float32(1e-39))).astype(np.float32).astype(BF16).view(np.uint16)
    assert np.mean(got == want) > 0.9999
    v = got.view(BF16).astype(np.float32)
    assert np.all(np.abs(v) < 2.0 ** -126) and np.mean(v != 0) > 0.95
