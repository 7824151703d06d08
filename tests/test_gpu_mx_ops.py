"""The mlx.core ops beyond the benchmark graphs (the rest of the reference
tracer's op set, ``ir/op_registry.py``) and the layer_norm / rope candidates
the reference's passes emit, on this backend against the oracle."""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from oracle import mlx_cpu
from phew_b200 import workloads as W

pytestmark = pytest.mark.gpu

SOURCES = Path(__file__).resolve().parent / "golden" / "sources"
TOL = {"float32": (1e-5, 1e-5), "bfloat16": (2e-2, 2e-2), "float16": (2e-3, 2e-3)}


def _load(key):
    ns: dict = {}
    exec(compile((SOURCES / f"{key}.py").read_text(), key, "exec"), ns)
    return ns["optimized"]


def _close(got, ref, dtype="float32"):
    g = np.asarray(got).astype(np.float64)
    r = np.asarray(ref).astype(np.float64)
    assert g.shape == r.shape, (g.shape, r.shape)
    rtol, atol = TOL[dtype]
    np.testing.assert_allclose(g, r, rtol=rtol, atol=atol)


def _rand(shape, dtype="float32", seed=0, scale=1.0):
    x = np.random.default_rng(seed).standard_normal(shape).astype(np.float32) * scale
    return x.astype(mlx_cpu._NP[dtype])


# --- candidates emitted by the reference's passes --------------------------

@pytest.mark.parametrize("key", ["layer_norm__fusion0", "layer_norm__fusion1"])
def test_layer_norm_candidates(mx, key):
    x, w, b = _rand((300, 2048), seed=1, scale=2), _rand((2048,), seed=2), _rand((2048,), seed=3)
    got = _load(key)(mx.array(x), mx.array(w), mx.array(b))
    ref = W.layer_norm_fn(mlx_cpu)(mlx_cpu.array(x), mlx_cpu.array(w), mlx_cpu.array(b))
    _close(got, ref)


def test_rope_candidate_with_fused_chain(mx):
    """rope__fusion1: the user's own rotation (cos / sin of the given angles),
    fused by the reference's fusion pass into one two-output kernel (whose
    output shapes the reference's emitter writes out at the traced shape,
    emit/codegen.py:538-582, so it runs at that shape)."""
    x = _rand((8, 32, 2048, 128), "bfloat16", seed=4)
    ang = (np.random.default_rng(5).uniform(-3, 3, (2048, 64))).astype(mlx_cpu._NP["bfloat16"])
    got = _load("rope__fusion1")(mx.array(x), mx.array(ang))
    ref = W.rope_fn(mlx_cpu)(mlx_cpu.array(x), mlx_cpu.array(ang))
    _close(got, ref, "bfloat16")


def test_rope_candidate_substituted(mx):
    """rope__fusion0: the substitution's FastRoPE (default base, positions
    0..L-1; the angle input is dropped, as the reference's rewrite drops it)."""
    x = _rand((2, 3, 512, 128), "bfloat16", seed=6)
    ang = np.zeros((512, 64), mlx_cpu._NP["bfloat16"])
    got = _load("rope__fusion0")(mx.array(x), mx.array(ang))
    ref = mlx_cpu.rope(mlx_cpu.array(x), 128)
    _close(got, ref, "bfloat16")


# --- reductions -------------------------------------------------------------

@pytest.mark.parametrize("dtype", ["float32", "bfloat16"])
@pytest.mark.parametrize("axis,keep", [(-1, True), (0, False), ((0, 2), False), (None, False)])
def test_var_std_logsumexp(mx, dtype, axis, keep):
    x = _rand((6, 50, 33), dtype, seed=7, scale=3)
    for name, kw in (("var", {}), ("var", {"ddof": 1}), ("std", {}), ("logsumexp", {})):
        got = getattr(mx, name)(mx.array(x), axis=axis, keepdims=keep, **kw)
        ref = getattr(mlx_cpu, name)(mlx_cpu.array(x), axis=axis, keepdims=keep, **kw)
        _close(got, ref, dtype)


def test_all_any_argmax_argmin(mx):
    x = _rand((7, 40), seed=8)
    x[2] = 0
    for name in ("all", "any"):
        got = getattr(mx, name)(mx.array(x), axis=1)
        ref = getattr(mlx_cpu, name)(mlx_cpu.array(x), axis=1)
        assert np.array_equal(np.asarray(got), np.asarray(ref))
    for name in ("argmax", "argmin"):
        with mx.allow_torch_kernels():
            got = getattr(mx, name)(mx.array(x), axis=1)
        ref = getattr(mlx_cpu, name)(mlx_cpu.array(x), axis=1)
        assert np.array_equal(np.asarray(got).astype(np.int64), np.asarray(ref).astype(np.int64))


# --- elementwise --------------------------------------------------------------

def test_float_classification_and_clip(mx):
    x = _rand((5, 64), seed=9, scale=3)
    x[0, :4] = [np.nan, np.inf, -np.inf, 0.0]
    for name in ("isnan", "isinf", "isfinite", "isposinf", "isneginf"):
        assert np.array_equal(np.asarray(getattr(mx, name)(mx.array(x))),
                              np.asarray(getattr(mlx_cpu, name)(mlx_cpu.array(x)))), name
    _close(mx.clip(mx.array(x[1:]), -1.0, 0.5), mlx_cpu.clip(mlx_cpu.array(x[1:]), -1.0, 0.5))
    y = np.asarray(mx.nan_to_num(mx.array(x)))
    assert np.isfinite(y).all() and y[0, 0] == 0


def test_bitwise_ops(mx):
    a = np.random.default_rng(10).integers(0, 1 << 20, (256,)).astype(np.int32)
    b = np.random.default_rng(11).integers(0, 1 << 20, (256,)).astype(np.int32)
    for name in ("bitwise_and", "bitwise_or", "bitwise_xor"):
        got = getattr(mx, name)(mx.array(a), mx.array(b))
        assert np.array_equal(np.asarray(got), getattr(np, name)(a, b)), name
    assert np.array_equal(np.asarray(mx.left_shift(mx.array(a), 3)), a << 3)
    assert np.array_equal(np.asarray(mx.right_shift(mx.array(a), 2)), a >> 2)
    assert np.array_equal(np.asarray(mx.bitwise_invert(mx.array(a))), ~a)


# --- assembly and layout -------------------------------------------------------

@pytest.mark.parametrize("dtype", ["float32", "bfloat16"])
def test_concatenate_stack_split_pad_tile_repeat_roll(mx, dtype):
    a, b = _rand((4, 6, 8), dtype, seed=12), _rand((4, 3, 8), dtype, seed=13)
    A, B = mx.array(a), mx.array(b)
    oa, ob = mlx_cpu.array(a), mlx_cpu.array(b)
    pairs = [
        (mx.concatenate([A, B], axis=1), mlx_cpu.concatenate([oa, ob], axis=1)),
        (mx.concatenate([A, A], axis=2), mlx_cpu.concatenate([oa, oa], axis=2)),
        (mx.concatenate([A, B], axis=None), mlx_cpu.concatenate([oa, ob], axis=None)),
        (mx.stack([A, A], axis=1), mlx_cpu.stack([oa, oa], axis=1)),
        (mx.pad(A, [(1, 2), (0, 0), (3, 1)], constant_values=1.5),
         mlx_cpu.pad(oa, [(1, 2), (0, 0), (3, 1)], constant_values=1.5)),
        (mx.tile(A, (2, 1, 3)), mlx_cpu.tile(oa, (2, 1, 3))),
        (mx.repeat(A, 3, axis=1), mlx_cpu.repeat(oa, 3, axis=1)),
        (mx.roll(A, 5, axis=2), mlx_cpu.roll(oa, 5, axis=2)),
        (mx.roll(A, -2), mlx_cpu.roll(oa, -2)),
        (mx.tril(A), mlx_cpu.tril(oa)), (mx.triu(A, 1), mlx_cpu.triu(oa, 1)),
        (mx.moveaxis(A, 0, 2), mlx_cpu.moveaxis(oa, 0, 2)),
        (mx.flatten(A, 1), mlx_cpu.flatten(oa, 1)),
        (mx.concatenate([mx.transpose(A, [0, 2, 1]), mx.transpose(B, [0, 2, 1])], axis=2),
         mlx_cpu.concatenate([mlx_cpu.transpose(oa, [0, 2, 1]), mlx_cpu.transpose(ob, [0, 2, 1])], axis=2)),
    ]
    for k, (g, r) in enumerate(pairs):
        assert np.array_equal(np.asarray(g), np.asarray(r)), k
    parts = mx.split(A, [2, 5], axis=1)
    refs = mlx_cpu.split(oa, [2, 5], axis=1)
    assert all(np.array_equal(np.asarray(p), np.asarray(r)) for p, r in zip(parts, refs))


def test_torch_kernel_ops_are_refused_without_opt_in(mx):
    x = mx.array(_rand((5, 30), seed=14))
    for fn in (lambda: mx.sort(x), lambda: mx.cumsum(x, axis=1), lambda: mx.topk(x, 2),
               lambda: mx.argmax(x), lambda: mx.einsum("ij->j", x)):
        with pytest.raises(NotImplementedError, match="torch's CUDA kernels"):
            fn()


def test_cumsum_sort_topk_take(mx):
    with mx.allow_torch_kernels():
        _cumsum_sort_topk_take(mx)


def _cumsum_sort_topk_take(mx):
    x = _rand((5, 30), seed=14)
    _close(mx.cumsum(mx.array(x), axis=1), mlx_cpu.cumsum(mlx_cpu.array(x), axis=1))
    _close(mx.cumsum(mx.array(x), axis=0, reverse=True, inclusive=False),
           mlx_cpu.cumsum(mlx_cpu.array(x), axis=0, reverse=True, inclusive=False))
    assert np.array_equal(np.asarray(mx.sort(mx.array(x), axis=1)), np.sort(x, axis=1))
    assert np.array_equal(np.asarray(mx.argsort(mx.array(x), axis=1)), np.argsort(x, axis=1, kind="stable"))
    assert np.array_equal(np.asarray(mx.topk(mx.array(x), 4, axis=1)),
                          np.asarray(mlx_cpu.topk(mlx_cpu.array(x), 4, axis=1)))
    idx = np.random.default_rng(15).integers(0, 30, (5, 7)).astype(np.int32)
    assert np.array_equal(np.asarray(mx.take_along_axis(mx.array(x), mx.array(idx), axis=1)),
                          np.take_along_axis(x, idx.astype(np.int64), 1))
    assert np.array_equal(np.asarray(mx.take(mx.array(x), mx.array(idx[0]), axis=1)),
                          np.take(x, idx[0].astype(np.int64), axis=1))


def test_hadamard_transform(mx):
    x = _rand((3, 64), seed=16)
    h = np.ones((1, 1), np.float32)
    while h.shape[0] < 64:
        h = np.block([[h, h], [h, -h]])
    _close(mx.hadamard_transform(mx.array(x)), (x @ h) / 8.0)


# --- group-wise quantised weights --------------------------------------------

@pytest.mark.parametrize("bits,group", [(4, 64), (8, 32), (2, 128)])
@pytest.mark.parametrize("dtype", ["bfloat16", "float16"])
def test_quantize_dequantize_and_quantized_matmul(mx, bits, group, dtype):
    w = _rand((256, 512), dtype, seed=bits + group, scale=0.05)
    wq, s, b = mx.quantize(mx.array(w), group_size=group, bits=bits)
    assert wq.shape == (256, 512 * bits // 32) and s.shape == (256, 512 // group)
    wd = mx.dequantize(wq, s, b, group_size=group, bits=bits)
    ref = mlx_cpu.dequantize(mlx_cpu.array(np.asarray(wq)), mlx_cpu.array(np.asarray(s)),
                             mlx_cpu.array(np.asarray(b)), group, bits)
    assert np.array_equal(np.asarray(wd).view(np.uint16), np.asarray(ref.v).view(np.uint16))
    # the codes reproduce w to within one quantisation step of its group
    step = np.repeat(np.asarray(s).astype(np.float32), group, axis=-1)
    err = np.abs(np.asarray(wd).astype(np.float32) - w.astype(np.float32))
    assert (err <= step * 0.5 + np.abs(w.astype(np.float32)) * 1e-2 + 1e-6).all()
    x = _rand((64, 512), dtype, seed=3)
    got = mx.quantized_matmul(mx.array(x), wq, s, b, transpose=True, group_size=group, bits=bits)
    refm = mlx_cpu.quantized_matmul(mlx_cpu.array(x), mlx_cpu.array(np.asarray(wq)),
                                    mlx_cpu.array(np.asarray(s)), mlx_cpu.array(np.asarray(b)),
                                    transpose=True, group_size=group, bits=bits)
    _close(got, refm, dtype)


def test_quantized_matmul_needs_scales(mx):
    """The reference's QuantizationPass emits quantized_matmul(x, W) without
    scales (rules/quantization.py:62-69); like MLX, that raises."""
    x = mx.array(_rand((4, 64), "bfloat16"))
    with pytest.raises(TypeError):
        mx.quantized_matmul(x, x, transpose=True)


def test_quantized_sdpa(mx):
    q = _rand((1, 2, 256, 128), "bfloat16", seed=20)
    k = _rand((1, 2, 256, 128), "bfloat16", seed=21)
    v = _rand((1, 2, 256, 128), "bfloat16", seed=22)
    kq, ks, kb = mx.quantize(mx.array(k), group_size=64, bits=8)
    vq, vs, vb = mx.quantize(mx.array(v), group_size=64, bits=8)
    # argument order of the emitted call (emit/codegen.py:428-435): q, k, v, then
    # scale_k, biases_k, scale_v, biases_v
    got = mx.fast.quantized_scaled_dot_product_attention(
        mx.array(q), kq, vq, ks, kb, vs, vb, scale=0.088, bits=8, group_size=64)
    kd = mlx_cpu.dequantize(mlx_cpu.array(np.asarray(kq)), mlx_cpu.array(np.asarray(ks)),
                            mlx_cpu.array(np.asarray(kb)), 64, 8)
    vd = mlx_cpu.dequantize(mlx_cpu.array(np.asarray(vq)), mlx_cpu.array(np.asarray(vs)),
                            mlx_cpu.array(np.asarray(vb)), 64, 8)
    ref = mlx_cpu.sdpa(mlx_cpu.array(q), kd, vd, 0.088)
    g = np.asarray(got).astype(np.float64)
    r = np.asarray(ref).astype(np.float64)
    assert np.abs(g - r).max() / np.sqrt(np.mean(np.asarray(vd.v).astype(np.float64) ** 2)) < 2e-2
