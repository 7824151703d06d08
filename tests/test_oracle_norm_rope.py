"""The oracle's layer_norm and rope restatements: identities they must
satisfy (no numeric goldens for these exist in the reference)."""

from __future__ import annotations

import numpy as np
import pytest

from oracle import mlx_cpu as m


def _x(shape, seed=0, dtype=np.float32):
    return m.array(np.random.default_rng(seed).standard_normal(shape).astype(dtype))


def test_rope_position_zero_is_identity_and_norms_are_kept():
    x = _x((2, 7, 32))
    y = np.asarray(m.rope(x, 32).v)
    xv = np.asarray(x.v)
    assert np.array_equal(y[:, 0], xv[:, 0])
    n0 = xv[..., :16] ** 2 + xv[..., 16:] ** 2
    n1 = y[..., :16] ** 2 + y[..., 16:] ** 2
    np.testing.assert_allclose(n1, n0, rtol=1e-5, atol=1e-6)


def test_rope_partial_dims_copy_the_tail():
    x = _x((3, 5, 24))
    y = np.asarray(m.rope(x, 8).v)
    assert np.array_equal(y[..., 8:], np.asarray(x.v)[..., 8:])
    assert np.array_equal(np.asarray(m.rope(x, 0).v), np.asarray(x.v))


def test_rope_traditional_is_the_interleaved_layout():
    x = _x((4, 6, 16), seed=1)
    xv = np.asarray(x.v)
    perm = np.concatenate([np.arange(0, 16, 2), np.arange(1, 16, 2)])  # interleaved -> halves
    a = np.asarray(m.rope(x, 16, traditional=True).v)[..., perm]
    b = np.asarray(m.rope(m.array(xv[..., perm]), 16).v)
    assert np.array_equal(a, b)


def test_rope_offset_is_a_shifted_sequence():
    x = _x((1, 12, 16), seed=2)
    full = np.asarray(m.rope(x, 16).v)
    tail = np.asarray(m.rope(m.array(np.asarray(x.v)[:, 5:]), 16, offset=5).v)
    assert np.array_equal(full[:, 5:], tail)


def test_layer_norm_standardises_and_applies_affine():
    x = _x((6, 64), seed=3)
    y = np.asarray(m.layer_norm(x).v).astype(np.float64)
    np.testing.assert_allclose(y.mean(-1), 0, atol=1e-6)
    np.testing.assert_allclose(y.var(-1), 1, rtol=1e-3)
    w = m.array(np.full(64, 2.0, np.float32))
    b = m.array(np.full(64, -1.0, np.float32))
    z = np.asarray(m.layer_norm(x, w, b).v)
    np.testing.assert_allclose(z, 2 * y - 1, rtol=1e-6, atol=1e-6)
    with pytest.raises(ValueError):
        m.layer_norm(x, m.array(np.ones(3, np.float32)))
