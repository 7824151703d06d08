"""The failure path of the tensor-core pipelines, made to run on purpose
without faulting the GPU: ``phew_test_inject_stall`` makes the next GEMM /
attention launch leave one producer load unissued and bounds its waits by
2 ms.  The consumers' waits run out, the call surfaces PHEW_ERR_TIMEOUT
through the error flag (``ops.check_device_errors``), and the next normal
launches on the same device -- on every SM, so also on the SMs whose
failed CTAs had to free their TMEM -- give the oracle's results."""

from __future__ import annotations

import ctypes
import math

import numpy as np
import pytest

from oracle import mlx_cpu

pytestmark = pytest.mark.gpu

BF16 = mlx_cpu.BF16
WAIT_NS = 2_000_000  # 2 ms


def _inject(stage: int) -> None:
    from phew_b200 import _native

    _native.call("phew_test_inject_stall", stage, ctypes.c_uint64(WAIT_NS))


def _rand(rng, shape, scale=1.0):
    return (rng.standard_normal(shape).astype(np.float32) * scale).astype(BF16)


def _expect_timeout(mx):
    from phew_b200 import _native
    from phew_b200.ops import check_device_errors

    mx.synchronize()
    with pytest.raises(_native.PhewError) as e:
        check_device_errors()
    assert e.value.status == _native.PHEW_ERR_TIMEOUT
    check_device_errors()  # the flag was cleared


def test_hook_rejects_bad_limits(mx):
    from phew_b200 import _native

    lib = _native.load()
    assert lib.phew_test_inject_stall(0, ctypes.c_uint64(0)) == _native.PHEW_ERR_INVALID
    assert lib.phew_test_inject_stall(0, ctypes.c_uint64(2 * 10**9)) == _native.PHEW_ERR_INVALID
    assert lib.phew_test_inject_stall(-1, ctypes.c_uint64(WAIT_NS)) == _native.PHEW_ERR_INVALID


def test_attention_wait_runs_out_then_recovers(mx):
    rng = np.random.default_rng(3)
    q, k, v = (_rand(rng, (1, 1, 256, 128)) for _ in range(3))
    _inject(0)  # V of key tile 0 never lands
    mx.fast.scaled_dot_product_attention(mx.array(q), mx.array(k), mx.array(v), scale=0.088)
    _expect_timeout(mx)
    # a launch with more CTAs than SMs, on fresh inputs, matches the oracle
    shape = (2, 16, 1024, 128)
    q, k, v = (_rand(rng, shape) for _ in range(3))
    got = np.asarray(mx.fast.scaled_dot_product_attention(
        mx.array(q), mx.array(k), mx.array(v), scale=1 / math.sqrt(128), mask="causal"))
    from phew_b200.ops import check_device_errors

    check_device_errors()
    vs = float(np.sqrt(np.mean(v.astype(np.float64) ** 2)))
    for bh in (0, 17, 31):
        b, h = divmod(bh, 16)
        ref = mlx_cpu.sdpa(*(mlx_cpu.array(a[b:b + 1, h:h + 1]) for a in (q, k, v)),
                           1 / math.sqrt(128), "causal")
        err = np.abs(got[b, h].astype(np.float64) - np.asarray(ref).astype(np.float64)[0, 0]).max()
        assert err / vs < 2e-2, (bh, err / vs)


def test_gemm_wait_runs_out_then_recovers(mx):
    rng = np.random.default_rng(4)
    a, b = _rand(rng, (256, 512)), _rand(rng, (512, 256), 1 / np.sqrt(512))
    _inject(2)  # the third k-block load of each CTA never lands
    mx.array(a) @ mx.array(b)
    _expect_timeout(mx)
    M, K, N = 4096, 1024, 4096  # 256 tiles: every SM runs one
    a, b = _rand(rng, (M, K)), _rand(rng, (K, N), 1 / np.sqrt(K))
    got = np.asarray(mx.array(a) @ mx.array(b))
    from phew_b200.ops import check_device_errors

    check_device_errors()
    rows = np.arange(0, M, 97)
    ref = (a[rows].astype(np.float32) @ b.astype(np.float32)).astype(BF16).astype(np.float64)
    g = got[rows].astype(np.float64)
    scale = float(np.sqrt(np.mean(ref * ref)))
    np.testing.assert_allclose(g, ref, rtol=2e-2, atol=2e-2 * scale)


def test_hook_is_one_shot(mx):
    """Only the next launch is affected: the one after it is clean."""
    rng = np.random.default_rng(5)
    a, b = _rand(rng, (256, 512)), _rand(rng, (512, 256), 1 / np.sqrt(512))
    _inject(1)
    mx.array(a) @ mx.array(b)
    _expect_timeout(mx)
    got = np.asarray(mx.array(a) @ mx.array(b)).astype(np.float64)
    from phew_b200.ops import check_device_errors

    check_device_errors()
    ref = (a.astype(np.float32) @ b.astype(np.float32)).astype(BF16).astype(np.float64)
    np.testing.assert_allclose(got, ref, rtol=2e-2, atol=2e-2 * float(np.sqrt(np.mean(ref * ref))))
