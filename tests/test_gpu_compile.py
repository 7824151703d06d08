"""mx.compile (deferred, fused elementwise groups) gives the same bits as
op-by-op evaluation, on the graphs the reference's candidates contain."""

from __future__ import annotations

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _same(mx, f, *args):
    eager = f(*args)
    fused = mx.compile(f)(*args)
    e = [np.asarray(x).view(np.uint8) for x in (eager if isinstance(eager, (list, tuple)) else [eager])]
    c = [np.asarray(x).view(np.uint8) for x in (fused if isinstance(fused, (list, tuple)) else [fused])]
    assert len(e) == len(c)
    for a, b in zip(e, c):
        assert a.shape == b.shape and np.array_equal(a, b)


def _rand(mx, rng, shape, dtype, scale=1.0):
    from oracle import mlx_cpu

    x = (rng.standard_normal(shape).astype(np.float32) * scale).astype(mlx_cpu._NP[dtype])
    return mx.array(x)


@pytest.mark.parametrize("dtype", ["bfloat16", "float16", "float32"])
def test_rms_norm_tail(mx, dtype):
    rng = np.random.default_rng(1)
    x = _rand(mx, rng, (2, 33, 256), dtype)
    w = _rand(mx, rng, (256,), dtype)

    def f(x, w):
        t = mx.mean(x * x, axis=[2], keepdims=True)
        return x * mx.rsqrt(t + mx.array(1e-5, dtype=getattr(mx, dtype))) * w

    _same(mx, f, x, w)


def test_attention_scores_scale_mask_softmax(mx):
    rng = np.random.default_rng(2)
    q = _rand(mx, rng, (2, 4, 256, 128), "bfloat16")
    k = _rand(mx, rng, (2, 4, 256, 128), "bfloat16")
    mask = mx.array(np.triu(np.full((256, 256), -1e9, np.float32), 1)).astype(mx.bfloat16)

    def f(q, k, mask):
        s = (q @ mx.transpose(k, [0, 1, 3, 2])) * mx.array(0.08838834764831843, dtype=mx.bfloat16)
        return mx.softmax(s + mask, axis=3)

    _same(mx, f, q, k, mask)


def test_swiglu_and_residual(mx):
    rng = np.random.default_rng(3)
    a = _rand(mx, rng, (64, 512), "bfloat16", 3)
    b = _rand(mx, rng, (64, 512), "bfloat16")
    r = _rand(mx, rng, (64, 1), "bfloat16")

    def f(a, b, r):
        g = a * r
        return g * mx.sigmoid(g) * (b * r), a + b

    _same(mx, f, a, b, r)


def test_gelu_chain_fp16(mx):
    rng = np.random.default_rng(4)
    x = _rand(mx, rng, (128, 1024), "float16")
    a = _rand(mx, rng, (1024,), "float16")
    c = _rand(mx, rng, (128, 1024), "float16")

    def f(x, a, c):
        y = x * a + 0.5
        g = 0.5 * y * (1.0 + mx.tanh(0.7978845608 * (y + 0.044715 * y * y * y)))
        return g * mx.sigmoid(c) + x

    _same(mx, f, x, a, c)


def test_mixed_dtypes_and_shared_terms(mx):
    rng = np.random.default_rng(5)
    h = _rand(mx, rng, (300,), "float16")
    s = _rand(mx, rng, (300,), "float32")

    def f(h, s):
        t = h + s
        return t * t - mx.exp(h * 0.1)

    _same(mx, f, h, s)


def test_pending_values_read_inside_the_function(mx):
    """Views, host reads and non-elementwise consumers force a pending value."""
    rng = np.random.default_rng(6)
    x = _rand(mx, rng, (8, 64), "bfloat16")

    def f(x):
        y = x * 2.0
        z = mx.reshape(y, [4, 128]) + 1.0
        total = float(np.asarray(mx.sum(y.astype(mx.float32))))
        return z * total

    _same(mx, f, x)


@pytest.mark.parametrize("dtype,cols", [("bfloat16", 256), ("bfloat16", 8192), ("bfloat16", 1000),
                                        ("bfloat16", 100), ("float16", 512), ("float32", 2048),
                                        ("float32", 36)])
def test_fused_softmax_matches_materialised(mx, dtype, cols):
    """softmax of a pending elementwise value runs as one kernel (prologue in
    registers) with the bits of materialise-then-softmax."""
    rng = np.random.default_rng(cols)
    s = _rand(mx, rng, (3, 7, cols), dtype, 3.0)
    m = np.zeros((7, cols), np.float32)
    m[2, cols // 3:] = -np.inf          # partly masked row
    m[4, :] = -np.inf                   # fully masked row: NaN, in both paths
    mask = mx.array(m).astype(getattr(mx, dtype))

    def f(s, mask):
        return mx.softmax(s * 0.125 + mask, axis=-1)

    _same(mx, f, s, mask)


@pytest.mark.parametrize("s_shape,m_shape,min_bytes", [((2, 4, 33, 512), (33, 512), 0),
                                                       ((2, 4, 5, 8192), (4, 5, 8192), 0),
                                                       ((3, 2, 9, 40), (9, 40), 0),
                                                       ((1, 3, 2048, 8192), (2048, 8192), None)])
def test_fused_softmax_shared_mask_rows(mx, monkeypatch, s_shape, m_shape, min_bytes):
    """Scores (B, H, L, cols) under a mask broadcast over the leading axes:
    the kernel hands rows out in mask-row order (every head's row q, then
    q + 1), with ragged last blocks; bits of materialise-then-softmax.  The
    small cases lower the mask-size bound so they take that order too; the
    last one (a 32 MiB mask) takes it at the default bound."""
    import phew_b200.emit.cuda_codegen as cg

    if min_bytes is not None:
        monkeypatch.setattr(cg, "SHARED_ROWS_MIN_BYTES", min_bytes)
    rng = np.random.default_rng(sum(s_shape))
    s = _rand(mx, rng, s_shape, "bfloat16", 3.0)
    m = np.triu(np.full(m_shape[-2:], -np.inf, np.float32), k=1)
    m = np.broadcast_to(m, m_shape) + rng.standard_normal(m_shape).astype(np.float32)
    mask = mx.array(np.ascontiguousarray(m)).astype(mx.bfloat16)

    def f(s, mask):
        return mx.softmax(s * 0.0883883 + mask, axis=-1)

    _same(mx, f, s, mask)


def test_fused_softmax_of_mixed_width_inputs_falls_back(mx):
    rng = np.random.default_rng(7)
    s = _rand(mx, rng, (4, 64), "float32")
    b = _rand(mx, rng, (64,), "bfloat16")

    def f(s, b):
        return mx.softmax((s + 1.0).astype(mx.bfloat16) * b, axis=-1)

    _same(mx, f, s, b)


@pytest.mark.parametrize("op", ["sum", "mean", "max", "min", "prod"])
@pytest.mark.parametrize("dtype,cols", [("bfloat16", 4096), ("float32", 2048), ("float16", 300),
                                        ("float32", 33)])
def test_fused_row_reduction_matches_materialised(mx, op, dtype, cols):
    """A reduction over the last axis of a pending elementwise value reads
    the prologue's inputs once, with the bits of materialise-then-reduce."""
    rng = np.random.default_rng(cols)
    x = _rand(mx, rng, (5, 9, cols), dtype)
    s = _rand(mx, rng, (5, 9, 1), dtype)
    if op == "max":
        xv = np.asarray(x).copy()
        xv[0, 0, 3] = np.nan
        x = mx.array(xv)

    def f(x, s):
        y = x * s + 0.25 if op != "prod" else 1.0 + x * 0.01
        return getattr(mx, op)(y, axis=-1, keepdims=(op == "mean")), getattr(mx, op)(y * y, axis=2)

    _same(mx, f, x, s)


def _row_maps(op=None):
    from phew_b200.mx import core

    return [k for k, v in core._kernel_cache.items()
            if isinstance(k, tuple) and k and k[0] == "row_map" and v and (op is None or k[1] == op)]


@pytest.mark.parametrize("dtype,shape", [("bfloat16", (4, 512, 4096)), ("float16", (3, 7, 1000)),
                                         ("float32", (5, 2048)), ("bfloat16", (4, 33, 96)),
                                         ("bfloat16", (2, 3, 4100)), ("float32", (7, 33))])
def test_row_map_rms_tail_one_kernel(mx, dtype, shape):
    """x * rsqrt(mean(x * x) + eps) * w: the reduction and the tail run as one
    row kernel, with the bits of op-by-op evaluation (vector and scalar
    forms, one and several rows per block, a partial last block)."""
    rng = np.random.default_rng(sum(shape))
    x = _rand(mx, rng, shape, dtype, 2.0)
    w = _rand(mx, rng, shape[-1:], dtype)
    before = len(_row_maps("mean"))

    def f(x, w):
        t = mx.mean(x * x, axis=[len(shape) - 1], keepdims=True)
        return x * mx.rsqrt(t + mx.array(1e-5, dtype=getattr(mx, dtype))) * w

    _same(mx, f, x, w)
    assert len(_row_maps("mean")) >= max(before, 1)


@pytest.mark.parametrize("op", ["max", "min", "sum", "prod"])
def test_row_map_other_reductions(mx, op):
    """x - op(x) and x * op(x) over rows, with NaN, signed zeros and a row of
    equal values (max / min keep the first of equal values, as the
    materialised reduction does)."""
    rng = np.random.default_rng(7)
    xv = (rng.standard_normal((6, 40, 300)).astype(np.float32)).astype(np.float16)
    xv[0, 0, 5] = np.nan
    xv[1, 1, :] = 0.0
    xv[1, 1, ::2] = -0.0
    xv[2, 2, :] = 1.5
    x = mx.array(xv)

    def f(x):
        y = x * 0.5 if op != "prod" else 1.0 + x * 0.001
        r = getattr(mx, op)(y, axis=-1, keepdims=True)
        return y - r, y * r

    _same(mx, f, x)
    assert _row_maps(op)


def test_row_map_layer_norm_and_plain_input(mx):
    """mean(x) of a plain input, x - mean, the variance and the tail: the
    variance and tail run as one row kernel after the mean."""
    rng = np.random.default_rng(11)
    x = _rand(mx, rng, (8, 64, 1024), "bfloat16", 3.0)
    w = _rand(mx, rng, (1024,), "bfloat16")
    b = _rand(mx, rng, (1024,), "bfloat16")

    def f(x, w, b):
        m = mx.mean(x, axis=-1, keepdims=True)
        d = x - m
        v = mx.mean(d * d, axis=-1, keepdims=True)
        return d * mx.rsqrt(v + 1e-5) * w + b

    _same(mx, f, x, w, b)


def test_deferred_reduction_read_elsewhere(mx):
    """A deferred row reduction that is returned, reshaped or read by a DAG
    over other rows is computed on its own, with the same bits."""
    rng = np.random.default_rng(12)
    x = _rand(mx, rng, (4, 16, 256), "bfloat16")
    z = _rand(mx, rng, (2, 4, 16, 256), "bfloat16")

    def f(x, z):
        m = mx.mean(x * x, axis=-1, keepdims=True)
        return m, mx.reshape(m, [4, 16]), z * m, x / m

    _same(mx, f, x, z)
