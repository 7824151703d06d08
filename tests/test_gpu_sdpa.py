"""Fused attention kernel against the oracle's SDPA (float32/float64 numpy),
and the attention candidates of the reference's rewrite on this backend."""

from __future__ import annotations

import math
from pathlib import Path

import numpy as np
import pytest

from oracle import mlx_cpu

pytestmark = pytest.mark.gpu

BF16 = mlx_cpu.BF16
SOURCES = Path(__file__).resolve().parent / "golden" / "sources"


@pytest.fixture(autouse=True)
def _no_device_errors(mx):
    from phew_b200.ops import check_device_errors

    yield
    mx.synchronize()
    check_device_errors()


def _qkv(rng, shape, dtype):
    return [rng.standard_normal(shape).astype(np.float32).astype(dtype) for _ in range(3)]


def check(got, ref, v=None):
    """Errors are measured against the scale of V: attention outputs are
    weighted means of V rows, and the kernel (like MLX's) rounds the softmax
    weights P to 16 bits before P @ V, an error of up to 2^-9 of |V| that does
    not shrink with the output's own magnitude."""
    g = np.asarray(got).astype(np.float64)
    r = np.asarray(ref).astype(np.float64)
    scale = np.sqrt(np.mean(np.asarray(v, np.float64) ** 2)) if v is not None else np.sqrt(np.mean(r * r))
    err = np.abs(g - r).max() / scale
    np.testing.assert_allclose(g, r, rtol=2e-2, atol=2e-2 * scale)
    assert err < 2e-2, err


@pytest.mark.parametrize("dtype", [BF16, np.float16])
@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("shape", [(1, 1, 128, 128), (1, 2, 384, 128), (2, 3, 512, 128),
                                   (1, 1, 640, 128), (1, 2, 1024, 128)])
def test_sdpa_fused(mx, dtype, causal, shape):
    rng = np.random.default_rng(shape[2] + causal)
    q, k, v = _qkv(rng, shape, dtype)
    scale = 1 / math.sqrt(shape[-1])
    mask = "causal" if causal else None
    got = mx.fast.scaled_dot_product_attention(mx.array(q), mx.array(k), mx.array(v), scale=scale,
                                               mask=mask)
    ref = mlx_cpu.sdpa(mlx_cpu.array(q), mlx_cpu.array(k), mlx_cpu.array(v), scale, mask)
    check(got, ref, v)


@pytest.mark.parametrize("dtype", [BF16, np.float16])
@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("B,T,H", [(2, 256, 3), (1, 512, 5)])
def test_sdpa_reads_fused_qkv_in_place(mx, dtype, causal, B, T, H):
    """q, k, v as (batch, head) views of a fused qkv projection
    (qkv.reshape(B, T, 3, H, D).transpose(2, 0, 3, 1, 4)): phew_sdpa_strided
    reads them through 4-D maps, with no copy."""
    from phew_b200 import _native

    D = 128
    rng = np.random.default_rng(T * H + causal)
    qkv = rng.standard_normal((B, T, 3 * H * D)).astype(np.float32).astype(dtype)
    x = mx.array(qkv).reshape(B, T, 3, H, D).transpose(2, 0, 3, 1, 4)
    q, k, v = x[0], x[1], x[2]
    mask = "causal" if causal else None
    n0 = _native.launch_count()
    got = mx.fast.scaled_dot_product_attention(q, k, v, scale=1 / math.sqrt(D), mask=mask)
    mx.synchronize()
    assert _native.launch_count() - n0 == 1  # the attention kernel alone
    o = qkv.reshape(B, T, 3, H, D).transpose(2, 0, 3, 1, 4)
    qn, kn, vn = (np.ascontiguousarray(o[i]) for i in range(3))
    ref = mlx_cpu.sdpa(mlx_cpu.array(qn), mlx_cpu.array(kn), mlx_cpu.array(vn), 1 / math.sqrt(D), mask)
    check(got, ref, vn)


def test_sdpa_large_logits(mx):
    """Rows whose maximum grows late exercise the lazy rescaling path."""
    rng = np.random.default_rng(5)
    shape = (1, 2, 512, 128)
    q, k, v = _qkv(rng, shape, BF16)
    k = (k.astype(np.float32) * np.linspace(0.1, 3.0, 512)[None, None, :, None]).astype(BF16)
    got = mx.fast.scaled_dot_product_attention(mx.array(q), mx.array(k), mx.array(v), scale=0.3,
                                               mask="causal")
    ref = mlx_cpu.sdpa(mlx_cpu.array(q), mlx_cpu.array(k), mlx_cpu.array(v), 0.3, "causal")
    check(got, ref, v)


def test_sdpa_nan_rows_and_keys(mx):
    """A NaN query element gives a NaN output row; a NaN key element poisons
    every row that sees that key (all rows without a mask, the rows at or
    after it with the causal mask)."""
    rng = np.random.default_rng(8)
    shape = (1, 2, 512, 128)
    for causal in (True, False):
        q, k, v = _qkv(rng, shape, BF16)
        q[0, 0, 37, 5] = np.nan
        k[0, 1, 300, 17] = np.nan
        mask = "causal" if causal else None
        got = np.asarray(mx.fast.scaled_dot_product_attention(
            mx.array(q), mx.array(k), mx.array(v), scale=1 / math.sqrt(128), mask=mask)).astype(np.float32)
        ref = np.asarray(mlx_cpu.sdpa(mlx_cpu.array(q), mlx_cpu.array(k), mlx_cpu.array(v),
                                      1 / math.sqrt(128), mask)).astype(np.float32)
        assert np.array_equal(np.isnan(got), np.isnan(ref))
        assert np.isnan(got[0, 0, 37]).all() and np.isfinite(got[0, 0, 36]).all()
        assert np.isnan(got[0, 1, 300]).all()
        assert np.isfinite(got[0, 1, 299]).all() == causal
        fin = np.isfinite(ref)
        check(np.where(fin, got, 0), np.where(fin, ref, 0), v)


def test_sdpa_nonpositive_scale_uses_composed_path(mx):
    rng = np.random.default_rng(9)
    shape = (1, 1, 256, 128)
    q, k, v = _qkv(rng, shape, BF16)
    # The composed path rounds the scores to bf16 before the softmax (as the
    # unsubstituted graph does); small |scale| keeps that rounding inside the
    # tolerance of the float32 oracle.
    for scale in (0.0, -0.05):
        got = mx.fast.scaled_dot_product_attention(mx.array(q), mx.array(k), mx.array(v), scale=scale,
                                                   mask="causal")
        ref = mlx_cpu.sdpa(mlx_cpu.array(q), mlx_cpu.array(k), mlx_cpu.array(v), scale, "causal")
        check(got, ref, v)


def test_sdpa_composed_fallback(mx):
    rng = np.random.default_rng(6)
    shape = (1, 2, 100, 64)  # not a multiple of 128, D = 64
    q, k, v = _qkv(rng, shape, BF16)
    got = mx.fast.scaled_dot_product_attention(mx.array(q), mx.array(k), mx.array(v), scale=0.125,
                                               mask="causal")
    ref = mlx_cpu.sdpa(mlx_cpu.array(q), mlx_cpu.array(k), mlx_cpu.array(v), 0.125, "causal")
    check(got, ref, v)


def _load(key):
    ns: dict = {}
    exec(compile((SOURCES / f"{key}.py").read_text(), key, "exec"), ns)
    return ns["optimized"]


def test_naive_attention_baseline_matches_oracle(mx):
    from phew_b200.workloads import WORKLOADS

    w = WORKLOADS["attention"]
    host = w.host_inputs("small", 0)
    host = [h[:1, :2] if h.ndim == 4 else h for h in host]
    got = w.make_fn(mx)(*[mx.array(h) for h in host])
    ref = mlx_cpu.sdpa(*[mlx_cpu.array(h) for h in host[:3]], 1 / math.sqrt(128), "causal")
    check(got, ref, host[2])


def test_sdpa_rewrite_drops_mask_and_is_rejected(mx):
    """The reference's SDPA substitution drops the causal mask
    (rules/primitive_subst.py:490-495); its candidate must fail verification
    against the masked baseline, as it does on the reference."""
    from phew_b200.verify import EquivalenceChecker
    from phew_b200.workloads import WORKLOADS

    w = WORKLOADS["attention"]
    cand = _load("attention__fusion0")
    base = w.make_fn(mx)

    def factory(size, seed):
        host = w.host_inputs("small", seed)
        return [mx.array(h[:1, :2] if h.ndim == 4 else h) for h in host], {}

    res = EquivalenceChecker(n_seeds=1, problem_sizes=["small"]).check(base, cand, factory)
    assert not res.passed
    assert any("variant=random" in f for f in res.failures)
