"""The rest of the ``mlx.core`` ops phew's tracer records (``ir/op_registry.py``
IMPLEMENTED), so harness functions and emitted sources that use them run here.

Where the work is elementwise it goes through the same emitted kernels as
every other elementwise op (and fuses inside ``mx.compile``); variance runs
on ``phew_reduce_var``; array assembly (concatenate, stack, pad, tile,
repeat, roll, slice_update) is views plus ``phew_copy_strided_to``.  Ops
that are data-dependent orderings or gathers (sort, argsort, topk,
partition, cumulative scans, take / take_along_axis / put_along_axis,
argmax / argmin, median, einsum) use torch's CUDA kernels on the same device
buffers.  They are off the candidate hot path (no candidate of the
verification sweep or the benchmark harnesses uses them), and because they
are not this backend's own kernels they raise ``NotImplementedError`` unless
the caller opts in: ``with allow_torch_kernels(): ...`` or
``PHEW_ALLOW_TORCH_KERNELS=1`` in the environment.
"""

from __future__ import annotations

import builtins
import contextlib
import ctypes
import math
import os
from typing import Any, Sequence

import numpy as np
import torch

from .. import _native
from .. import dtypes as dt
from .core import (
    _elementwise,
    _norm_axes,
    _numel,
    _reduce,
    _stream,
    array,
    asarray_device,
    astype,
    broadcast_to,
    contiguous_copy,
    device,
    empty,
    expand_dims,
    reshape,
    transpose,
    where,
)

__all__ = [
    "isnan", "isinf", "isfinite", "isposinf", "isneginf", "bitwise_and", "bitwise_or",
    "bitwise_xor", "bitwise_invert", "left_shift", "right_shift", "clip", "nan_to_num", "conj",
    "conjugate", "real", "imag", "divmod", "var", "std", "logsumexp", "all", "any", "argmax",
    "argmin", "cumsum", "cumprod", "cummax", "cummin", "logcumsumexp", "sort", "argsort", "topk",
    "partition", "argpartition", "median", "take", "take_along_axis", "put_along_axis", "arange",
    "linspace", "eye", "identity", "tri", "tril", "triu", "meshgrid", "diag", "diagonal", "trace",
    "concatenate", "concat", "stack", "split", "pad", "tile", "repeat", "roll", "moveaxis",
    "permute_dims", "flatten", "unflatten", "atleast_1d", "atleast_2d", "atleast_3d",
    "contiguous", "view", "as_strided", "slice", "slice_update", "asarray", "einsum",
    "allow_torch_kernels",
    "hadamard_transform", "bartlett", "blackman", "hamming", "hanning", "quantize", "dequantize",
    "quantized_matmul",
]


def quantize(w, group_size: int = 64, bits: int = 4, **_):
    from ..ops import quantize as _q

    return _q(w, group_size, bits)


def dequantize(w, scales, biases, group_size: int = 64, bits: int = 4, **_):
    from ..ops import dequantize as _dq

    return _dq(w, scales, biases, group_size, bits)


def quantized_matmul(x, w, scales=None, biases=None, transpose: bool = True, group_size: int = 64,
                     bits: int = 4, **_):
    from ..ops import quantized_matmul as _qmm

    return _qmm(x, w, scales, biases, transpose=transpose, group_size=group_size, bits=bits)


# Ops that run on torch's CUDA kernels instead of this library's: refused
# unless the caller opts in (see the module docstring).
_TORCH_KERNELS = {"on": os.environ.get("PHEW_ALLOW_TORCH_KERNELS", "") == "1"}


@contextlib.contextmanager
def allow_torch_kernels(flag: bool = True):
    """Within the block, ops backed by torch's CUDA kernels (sorts, scans,
    gathers, argmax / argmin, median, einsum) may run."""
    prev = _TORCH_KERNELS["on"]
    _TORCH_KERNELS["on"] = bool(flag)
    try:
        yield
    finally:
        _TORCH_KERNELS["on"] = prev


def _torch_kernel_op(name: str) -> None:
    if not _TORCH_KERNELS["on"]:
        raise NotImplementedError(
            f"mx.{name} runs on torch's CUDA kernels, not on this backend's own; it is off the "
            "candidate path.  Opt in with `with phew_b200.mx.allow_torch_kernels():` or "
            "PHEW_ALLOW_TORCH_KERNELS=1")


def _arr(x) -> array:
    return x if isinstance(x, array) else array(x)


def _wrap(t: torch.Tensor) -> array:
    return array._wrap(t)


# ---------------------------------------------------------------------------
# elementwise (emitted kernels)
# ---------------------------------------------------------------------------

def _pred(op):
    def f(a, *_, **__):
        return _elementwise(op, [_arr(a)], out_bool=True)

    f.__name__ = op
    return f


isnan = _pred("isnan")
isinf = _pred("isinf")
isfinite = _pred("isfinite")
isposinf = _pred("isposinf")
isneginf = _pred("isneginf")


def _bit(op):
    def f(a, b, *_, **__):
        return _elementwise(op, [a, b])

    f.__name__ = op
    return f


bitwise_and = _bit("bitwise_and")
bitwise_or = _bit("bitwise_or")
bitwise_xor = _bit("bitwise_xor")
left_shift = _bit("left_shift")
right_shift = _bit("right_shift")


def bitwise_invert(a, *_, **__):
    return _elementwise("bitwise_invert", [_arr(a)])


def clip(a, a_min=None, a_max=None, **_):
    """min(max(a, a_min), a_max) with None bounds omitted (mx.clip)."""
    out = _arr(a)
    if a_min is not None:
        out = _elementwise("maximum", [out, a_min])
    if a_max is not None:
        out = _elementwise("minimum", [out, a_max])
    return out


def nan_to_num(a, nan: float = 0.0, posinf: float | None = None, neginf: float | None = None, **_):
    """NaN -> `nan`, +inf -> `posinf`, -inf -> `neginf` (default: the dtype's
    largest finite values), as mx.nan_to_num."""
    a = _arr(a)
    if a.dtype.kind != "f":
        return a
    fmax = float(torch.finfo(a.dtype.torch).max)
    hi = fmax if posinf is None else posinf
    lo = -fmax if neginf is None else neginf
    out = where(isnan(a), nan, a)
    out = where(isposinf(a), hi, out)
    return where(isneginf(a), lo, out)


def conj(a, **_):
    """Real dtypes only on this backend: the identity."""
    return _arr(a)


conjugate = conj


def real(a, **_):
    return _arr(a)


def imag(a, **_):
    a = _arr(a)
    return _wrap(torch.zeros(a.shape, dtype=a.dtype.torch, device=device()))


def divmod(a, b, **_):  # noqa: A001  (MLX name)
    return _elementwise("floor_divide", [a, b]), _elementwise("remainder", [a, b])


# ---------------------------------------------------------------------------
# reductions
# ---------------------------------------------------------------------------

def _layout(a: array, axis, keepdims: bool):
    """(contiguous source, outer, red, inner, output shape) for reducing
    `axis` of `a` as [outer, red, inner] (axes moved together first)."""
    axes = _norm_axes(a, axis)
    shape = a.shape
    keep = tuple(1 if i in axes else s for i, s in enumerate(shape))
    out_shape = keep if keepdims else tuple(s for i, s in enumerate(shape) if i not in axes)
    src = asarray_device(a)
    if axes and axes != tuple(range(axes[0], axes[-1] + 1)):
        rest = [i for i in range(a.ndim) if i not in axes]
        src = contiguous_copy(transpose(src, rest + list(axes)))
        shape = tuple(a.shape[i] for i in rest) + tuple(a.shape[i] for i in axes)
        axes = tuple(range(len(rest), a.ndim))
    if not axes:
        return src, _numel(shape), 1, 1, out_shape
    return (src, _numel(shape[: axes[0]]), _numel(shape[axes[0]: axes[-1] + 1]),
            _numel(shape[axes[-1] + 1:]), out_shape)


def var(a, axis=None, keepdims: bool = False, ddof: int = 0, **_):
    """mx.var: fp32 mean, fp32 sum of squared deviations / (n - ddof),
    rounded once (``phew_reduce_var``)."""
    a = _arr(a)
    if a.dtype.code is None:
        a = astype(a, dt.float32)
    src, outer, red, inner, out_shape = _layout(a, axis, keepdims)
    out = empty(out_shape, a.dtype)
    if out.size == 0:
        return out
    if red == 0:
        out._t.fill_(float("nan"))
        return out
    _native.call("phew_reduce_var", ctypes.c_void_p(src._t.data_ptr()), ctypes.c_void_p(out._t.data_ptr()),
                 outer, red, inner, int(ddof), a.dtype.code, _stream())
    return out


def std(a, axis=None, keepdims: bool = False, ddof: int = 0, **_):
    """mx.std: sqrt of mx.var (two roundings, as MLX composes it)."""
    return _elementwise("sqrt", [var(a, axis, keepdims, ddof)])


def logsumexp(a, axis=None, keepdims: bool = False, **_):
    """log(sum(exp(a - m))) + m with m the (finite-guarded) max, in fp32 and
    rounded once to a's dtype."""
    a = _arr(a)
    x = astype(a, dt.float32) if a.dtype is not dt.float32 else a
    m = _reduce("max", x, axis, True)
    m = where(isinf(m), 0.0, m)
    s = _reduce("sum", _elementwise("exp", [_elementwise("sub", [x, m])]), axis, True)
    r = _elementwise("add", [_elementwise("log", [s]), m])
    if not keepdims:
        r = reshape(r, [d for i, d in enumerate(r.shape) if i not in _norm_axes(x, axis)])
    return astype(r, a.dtype) if a.dtype is not dt.float32 else r


def _as_float(a: array) -> array:
    return astype(_elementwise("ne", [a, 0], out_bool=True), dt.float32)


def all(a, axis=None, keepdims: bool = False, **_):  # noqa: A001
    return astype(_reduce("min", _as_float(_arr(a)), axis, keepdims), dt.bool_)


def any(a, axis=None, keepdims: bool = False, **_):  # noqa: A001
    return astype(_reduce("max", _as_float(_arr(a)), axis, keepdims), dt.bool_)


def _axis_arg(a: array, axis):
    return None if axis is None else int(axis) % builtins.max(a.ndim, 1)


def argmax(a, axis=None, keepdims: bool = False, **_):
    """Index of the first maximum, uint32 (torch CUDA; off the hot path)."""
    _torch_kernel_op("argmax")
    a = _arr(a)
    t = a._t.argmax() if axis is None else a._t.argmax(dim=_axis_arg(a, axis), keepdim=keepdims)
    return _wrap(t.to(torch.int32).view(torch.uint32) if hasattr(torch, "uint32") else t.to(torch.int32))


def argmin(a, axis=None, keepdims: bool = False, **_):
    """Index of the first minimum, uint32 (torch CUDA; off the hot path)."""
    _torch_kernel_op("argmin")
    a = _arr(a)
    t = a._t.argmin() if axis is None else a._t.argmin(dim=_axis_arg(a, axis), keepdim=keepdims)
    return _wrap(t.to(torch.int32).view(torch.uint32) if hasattr(torch, "uint32") else t.to(torch.int32))


def _scan(fn, a, axis, reverse, inclusive):
    _torch_kernel_op(fn.__name__.lstrip("_"))
    a = _arr(a)
    t = a._t.reshape(-1) if axis is None else a._t
    ax = 0 if axis is None else int(axis) % a.ndim
    if reverse:
        t = t.flip(ax)
    r = fn(t, ax)
    if not inclusive:
        r = torch.roll(r, 1, ax)
        idx = [builtins.slice(None)] * r.dim()
        idx[ax] = 0
        r[tuple(idx)] = _scan_identity(fn, r.dtype)
    if reverse:
        r = r.flip(ax)
    return _wrap(r.contiguous())


def _scan_identity(fn, d):
    if fn is _cumsum:
        return 0
    if fn is _cumprod:
        return 1
    if fn is _logcumsumexp:
        return -math.inf
    info = torch.finfo(d) if d.is_floating_point else torch.iinfo(d)
    return info.min if fn is _cummax else info.max


def _cumsum(t, ax):
    return torch.cumsum(t.float() if t.dtype in (torch.float16, torch.bfloat16) else t, ax).to(t.dtype)


def _cumprod(t, ax):
    return torch.cumprod(t.float() if t.dtype in (torch.float16, torch.bfloat16) else t, ax).to(t.dtype)


def _cummax(t, ax):
    return torch.cummax(t, ax).values


def _cummin(t, ax):
    return torch.cummin(t, ax).values


def _logcumsumexp(t, ax):
    return torch.logcumsumexp(t.float(), ax).to(t.dtype)


def cumsum(a, axis=None, reverse: bool = False, inclusive: bool = True, **_):
    """Scan (torch CUDA, fp32 accumulation; off the hot path)."""
    return _scan(_cumsum, a, axis, reverse, inclusive)


def cumprod(a, axis=None, reverse: bool = False, inclusive: bool = True, **_):
    return _scan(_cumprod, a, axis, reverse, inclusive)


def cummax(a, axis=None, reverse: bool = False, inclusive: bool = True, **_):
    return _scan(_cummax, a, axis, reverse, inclusive)


def cummin(a, axis=None, reverse: bool = False, inclusive: bool = True, **_):
    return _scan(_cummin, a, axis, reverse, inclusive)


def logcumsumexp(a, axis=None, reverse: bool = False, inclusive: bool = True, **_):
    return _scan(_logcumsumexp, a, axis, reverse, inclusive)


# ---------------------------------------------------------------------------
# orderings and gathers (torch CUDA kernels; off the candidate hot path)
# ---------------------------------------------------------------------------

def _flat_or_axis(a: array, axis):
    if axis is None:
        return a._t.reshape(-1), 0
    return a._t, int(axis) % a.ndim


def sort(a, axis=-1, **_):
    _torch_kernel_op("sort")
    t, ax = _flat_or_axis(_arr(a), axis)
    return _wrap(torch.sort(t, dim=ax, stable=True).values.contiguous())


def argsort(a, axis=-1, **_):
    _torch_kernel_op("argsort")
    t, ax = _flat_or_axis(_arr(a), axis)
    return _wrap(torch.sort(t, dim=ax, stable=True).indices.to(torch.int32).contiguous())


def partition(a, kth: int, axis=-1, **_):
    """A full sort satisfies the partition contract (k-th element in place,
    smaller ones before it, larger after)."""
    return sort(a, axis)


def argpartition(a, kth: int, axis=-1, **_):
    return argsort(a, axis)


def topk(a, k: int, axis=-1, **_):
    """The k largest values along `axis` (ascending, as MLX returns them)."""
    _torch_kernel_op("topk")
    t, ax = _flat_or_axis(_arr(a), axis)
    v = torch.topk(t, int(k), dim=ax, largest=True, sorted=True).values
    return _wrap(v.flip(ax).contiguous())


def median(a, axis=None, keepdims: bool = False, **_):
    """Mean of the two middle values for even counts (MLX's definition)."""
    _torch_kernel_op("median")
    a = _arr(a)
    x = astype(a, dt.float32)
    axes = _norm_axes(x, axis)
    rest = [i for i in range(x.ndim) if i not in axes]
    t = x._t.permute(*rest, *axes).reshape(*[x.shape[i] for i in rest], -1)
    s = torch.sort(t, dim=-1).values
    n = s.shape[-1]
    m = (s[..., (n - 1) // 2] + s[..., n // 2]) * 0.5
    if keepdims:
        m = m.reshape([1 if i in axes else d for i, d in enumerate(x.shape)])
    return astype(_wrap(m.contiguous()), a.dtype)


def take(a, indices, axis=None, **_):
    _torch_kernel_op("take")
    a = _arr(a)
    idx = _arr(indices)._t.long()
    if axis is None:
        return _wrap(a._t.reshape(-1)[idx].contiguous())
    ax = int(axis) % a.ndim
    return _wrap(torch.index_select(a._t, ax, idx.reshape(-1)).reshape(
        *a.shape[:ax], *idx.shape, *a.shape[ax + 1:]).contiguous())


def take_along_axis(a, indices, axis=None, **_):
    _torch_kernel_op("take_along_axis")
    a = _arr(a)
    idx = _arr(indices)._t.long()
    if axis is None:
        return _wrap(a._t.reshape(-1).gather(0, idx.reshape(-1)).contiguous())
    ax = int(axis) % a.ndim
    shape = torch.broadcast_shapes(tuple(a.shape[:ax]) + (idx.shape[ax],) + tuple(a.shape[ax + 1:]),
                                   tuple(idx.shape))
    src_shape = list(shape)
    src_shape[ax] = a.shape[ax]
    return _wrap(torch.gather(a._t.expand(src_shape), ax, idx.expand(shape)).contiguous())


def put_along_axis(a, indices, values, axis=None, **_):
    _torch_kernel_op("put_along_axis")
    a = _arr(a)
    out = a._t.clone()
    idx = _arr(indices)._t.long()
    v = _arr(values)._t.to(out.dtype)
    if axis is None:
        flat = out.reshape(-1)
        flat.scatter_(0, idx.reshape(-1), v.expand(idx.shape).reshape(-1))
        return _wrap(flat.reshape(out.shape))
    ax = int(axis) % a.ndim
    out.scatter_(ax, idx.expand_as(v) if v.dim() == idx.dim() else idx, v.expand(idx.shape))
    return _wrap(out)


def einsum(subscripts: str, *operands, **_):
    """torch.einsum on the device buffers (cuBLAS for contractions; no
    candidate on the sweep's hot path emits einsum)."""
    _torch_kernel_op("einsum")
    ts = [_arr(x)._t for x in operands]
    return _wrap(torch.einsum(subscripts, *ts).contiguous())


# ---------------------------------------------------------------------------
# constructors
# ---------------------------------------------------------------------------

def _dtype_or(dtype, default):
    return dt.from_any(dtype) if dtype is not None else default


def arange(*args, dtype=None, **kw):
    """mx.arange(stop) / arange(start, stop[, step])."""
    start, stop, step = 0, None, 1
    if "start" in kw:
        start = kw["start"]
    if "stop" in kw:
        stop = kw["stop"]
    if "step" in kw:
        step = kw["step"]
    if len(args) == 1:
        stop = args[0]
    elif len(args) == 2:
        start, stop = args
    elif len(args) >= 3:
        start, stop, step = args[:3]
    is_float = builtins.any(isinstance(v, float) for v in (start, stop, step))
    d = _dtype_or(dtype, dt.float32 if is_float else dt.int32)
    n = builtins.max(0, math.ceil((stop - start) / step))
    vals = np.asarray(start + step * np.arange(n, dtype=np.float64), dtype=np.float64)
    return array(vals.astype(np.float32) if d.kind == "f" else vals.astype(np.int64), d)


def linspace(start, stop, num: int = 50, dtype=None, **_):
    d = _dtype_or(dtype, dt.float32)
    return array(np.linspace(start, stop, int(num), dtype=np.float64).astype(np.float32), d)


def eye(n: int, m: int | None = None, k: int = 0, dtype=None, **_):
    d = _dtype_or(dtype, dt.float32)
    return array(np.eye(int(n), None if m is None else int(m), int(k), dtype=np.float32), d)


def identity(n: int, dtype=None, **_):
    return eye(n, dtype=dtype)


def tri(n: int, m: int | None = None, k: int = 0, dtype=None, **_):
    d = _dtype_or(dtype, dt.float32)
    return array(np.tri(int(n), None if m is None else int(m), int(k), dtype=np.float32), d)


def tril(x, k: int = 0, **_):
    """Zero above the k-th diagonal of the last two axes (a mask multiply in
    the emitted elementwise kernel)."""
    x = _arr(x)
    n, m = x.shape[-2], x.shape[-1]
    mask = array(np.tri(n, m, int(k), dtype=bool), dt.bool_)
    return where(mask, x, _zero(x))


def triu(x, k: int = 0, **_):
    x = _arr(x)
    n, m = x.shape[-2], x.shape[-1]
    mask = array(~np.tri(n, m, int(k) - 1, dtype=bool), dt.bool_)
    return where(mask, x, _zero(x))


def _zero(x: array):
    return 0 if x.dtype.kind == "f" else 0


def meshgrid(*arrays, sparse: bool = False, indexing: str = "xy", **_):
    ts = [_arr(a)._t for a in arrays]
    grids = torch.meshgrid(*ts, indexing=indexing)
    if sparse:
        out = []
        for i, t in enumerate(ts):
            shape = [1] * len(ts)
            j = i
            if indexing == "xy" and len(ts) >= 2 and i < 2:
                j = 1 - i
            shape[j] = t.numel()
            out.append(_wrap(t.reshape(shape).contiguous()))
        return out
    return [_wrap(g.contiguous()) for g in grids]


def diag(a, k: int = 0, **_):
    a = _arr(a)
    return _wrap(torch.diag(a._t, int(k)).contiguous())


def diagonal(a, offset: int = 0, axis1: int = 0, axis2: int = 1, **_):
    a = _arr(a)
    return _wrap(torch.diagonal(a._t, int(offset), int(axis1), int(axis2)).contiguous())


def trace(a, offset: int = 0, axis1: int = 0, axis2: int = 1, dtype=None, **_):
    d = diagonal(a, offset, axis1, axis2)
    from .core import sum as _sum

    r = _sum(d, axis=-1)
    return astype(r, dtype) if dtype is not None else r


def _window(fn):
    def f(M: int, **_):
        return array(fn(int(M)).astype(np.float32), dt.float32)

    return f


bartlett = _window(np.bartlett)
blackman = _window(np.blackman)
hamming = _window(np.hamming)
hanning = _window(np.hanning)


# ---------------------------------------------------------------------------
# assembly: views + phew_copy_strided_to
# ---------------------------------------------------------------------------

def _copy_into(dst: torch.Tensor, src: torch.Tensor) -> None:
    """dst[...] = src for two same-shape tensors with any strides (dst a view
    of a larger buffer), through phew_copy_strided_to."""
    if src.numel() == 0:
        return
    if src.dtype != dst.dtype:
        src = astype(_wrap(src), dt.from_any(dst.dtype))._t
    shape = list(dst.shape) or [1]
    if len(shape) > 8:
        raise NotImplementedError("copies of more than 8 dimensions")
    s_str = list(src.stride()) or [1]
    d_str = list(dst.stride()) or [1]
    n = len(shape)
    arr_t = ctypes.c_int64 * n
    _native.call(
        "phew_copy_strided_to", ctypes.c_void_p(src.data_ptr()), ctypes.c_void_p(dst.data_ptr()), n,
        arr_t(*shape), arr_t(*s_str), arr_t(*d_str), src.element_size(), _stream(),
    )


def concatenate(arrays: Sequence[Any], axis: int | None = 0, **_):
    arrs = [_arr(a) for a in arrays]
    if axis is None:
        arrs = [reshape(a, [-1]) for a in arrs]
        axis = 0
    res = arrs[0].dtype
    for a in arrs[1:]:
        res = dt.promote(res, a.dtype)
    nd = arrs[0].ndim
    ax = int(axis) % nd
    shape = list(arrs[0].shape)
    shape[ax] = builtins.sum(a.shape[ax] for a in arrs)
    out = empty(shape, res)
    off = 0
    for a in arrs:
        n = a.shape[ax]
        idx = [builtins.slice(None)] * nd
        idx[ax] = builtins.slice(off, off + n)
        _copy_into(out._t[tuple(idx)], a._t)
        off += n
    return out


concat = concatenate


def stack(arrays: Sequence[Any], axis: int = 0, **_):
    arrs = [_arr(a) for a in arrays]
    ax = int(axis) % (arrs[0].ndim + 1)
    return concatenate([expand_dims(a, ax) for a in arrs], axis=ax)


def split(a, indices_or_sections, axis: int = 0, **_):
    a = _arr(a)
    ax = int(axis) % a.ndim
    n = a.shape[ax]
    if isinstance(indices_or_sections, int):
        k = indices_or_sections
        if n % k:
            raise ValueError(f"split: {n} elements do not divide into {k} equal sections")
        cuts = [n // k * i for i in range(1, k)]
    else:
        cuts = [int(i) for i in indices_or_sections]
    bounds = [0] + cuts + [n]
    out = []
    for lo, hi in zip(bounds[:-1], bounds[1:]):
        idx = [builtins.slice(None)] * a.ndim
        idx[ax] = builtins.slice(lo, hi)
        out.append(_wrap(a._t[tuple(idx)]))
    return out


def pad(a, pad_width, mode: str = "constant", constant_values=0, **_):
    """Constant padding (mx.pad's default mode)."""
    a = _arr(a)
    if mode != "constant":
        raise NotImplementedError(f"pad mode {mode!r}")
    if isinstance(pad_width, int):
        pw = [(pad_width, pad_width)] * a.ndim
    elif len(pad_width) and isinstance(pad_width[0], int):
        pw = [tuple(pad_width)] * a.ndim if len(pad_width) == 2 else [(p, p) for p in pad_width]
    else:
        pw = [tuple(p) for p in pad_width]
        if len(pw) == 1:
            pw = pw * a.ndim
    shape = [s + lo + hi for s, (lo, hi) in zip(a.shape, pw)]
    cv = float(_arr(constant_values).item()) if isinstance(constant_values, array) else constant_values
    out = _wrap(torch.full(shape, cv, dtype=a.dtype.torch, device=device()))
    idx = tuple(builtins.slice(lo, lo + s) for (lo, _), s in zip(pw, a.shape))
    _copy_into(out._t[idx], a._t)
    return out


def tile(a, reps, **_):
    a = _arr(a)
    reps = [reps] if isinstance(reps, int) else list(reps)
    nd = builtins.max(a.ndim, len(reps))
    reps = [1] * (nd - len(reps)) + reps
    x = reshape(a, [1] * (nd - a.ndim) + list(a.shape))
    # [r0, s0, r1, s1, ...] broadcast view, then one strided copy
    view_shape, expand = [], []
    for r, s in zip(reps, x.shape):
        view_shape += [1, s]
        expand += [r, s]
    v = _wrap(x._t.reshape(view_shape).expand(expand))
    return reshape(contiguous_copy(v), [r * s for r, s in zip(reps, x.shape)])


def repeat(a, repeats: int, axis: int | None = None, **_):
    a = _arr(a)
    if axis is None:
        a = reshape(a, [-1])
        axis = 0
    ax = int(axis) % a.ndim
    shape = list(a.shape)
    v = _wrap(a._t.unsqueeze(ax + 1).expand(*shape[: ax + 1], int(repeats), *shape[ax + 1:]))
    shape[ax] *= int(repeats)
    return reshape(contiguous_copy(v), shape)


def roll(a, shift, axis=None, **_):
    a = _arr(a)
    if axis is None:
        flat = reshape(a, [-1])
        return reshape(roll(flat, shift, 0), list(a.shape))
    shifts = [shift] if isinstance(shift, int) else list(shift)
    axes = [axis] if isinstance(axis, int) else list(axis)
    out = a
    for s, ax in zip(shifts, axes):
        ax = int(ax) % out.ndim
        n = out.shape[ax]
        if n == 0:
            continue
        s = int(s) % n
        if s == 0:
            continue
        res = empty(out.shape, out.dtype)
        idx_src_hi = [builtins.slice(None)] * out.ndim
        idx_src_lo = [builtins.slice(None)] * out.ndim
        idx_dst_lo = [builtins.slice(None)] * out.ndim
        idx_dst_hi = [builtins.slice(None)] * out.ndim
        idx_src_hi[ax] = builtins.slice(n - s, n)
        idx_dst_lo[ax] = builtins.slice(0, s)
        idx_src_lo[ax] = builtins.slice(0, n - s)
        idx_dst_hi[ax] = builtins.slice(s, n)
        _copy_into(res._t[tuple(idx_dst_lo)], out._t[tuple(idx_src_hi)])
        _copy_into(res._t[tuple(idx_dst_hi)], out._t[tuple(idx_src_lo)])
        out = res
    return out


def moveaxis(a, source: int, destination: int, **_):
    a = _arr(a)
    return _wrap(torch.movedim(a._t, int(source), int(destination)))


def permute_dims(a, axes=None, **_):
    return transpose(_arr(a), axes)


def flatten(a, start_axis: int = 0, end_axis: int = -1, **_):
    a = _arr(a)
    if a.ndim == 0:
        return reshape(a, [1])
    s = int(start_axis) % a.ndim
    e = int(end_axis) % a.ndim
    shape = list(a.shape[:s]) + [_numel(a.shape[s: e + 1])] + list(a.shape[e + 1:])
    return reshape(a, shape)


def unflatten(a, axis: int, shape, **_):
    a = _arr(a)
    ax = int(axis) % a.ndim
    shape = list(shape)
    if -1 in shape:
        known = _numel([s for s in shape if s != -1])
        shape[shape.index(-1)] = a.shape[ax] // builtins.max(known, 1)
    return reshape(a, list(a.shape[:ax]) + shape + list(a.shape[ax + 1:]))


def atleast_1d(*arrays, **_):
    out = [reshape(_arr(a), [1]) if _arr(a).ndim == 0 else _arr(a) for a in arrays]
    return out[0] if len(out) == 1 else out


def atleast_2d(*arrays, **_):
    out = []
    for a in arrays:
        a = _arr(a)
        out.append(reshape(a, [1] * (2 - a.ndim) + list(a.shape)) if a.ndim < 2 else a)
    return out[0] if len(out) == 1 else out


def atleast_3d(*arrays, **_):
    out = []
    for a in arrays:
        a = _arr(a)
        if a.ndim == 0:
            out.append(reshape(a, [1, 1, 1]))
        elif a.ndim == 1:
            out.append(reshape(a, [1, a.shape[0], 1]))
        elif a.ndim == 2:
            out.append(reshape(a, list(a.shape) + [1]))
        else:
            out.append(a)
    return out[0] if len(out) == 1 else out


def contiguous(a, allow_col_major: bool = False, **_):
    return asarray_device(_arr(a))


def view(a, dtype, **_):
    """Reinterpret the bytes as `dtype` (same itemsize, or a divisible last axis)."""
    a = asarray_device(_arr(a))
    return _wrap(a._t.view(dt.from_any(dtype).torch))


def as_strided(a, shape=None, strides=None, offset: int = 0, **_):
    a = asarray_device(_arr(a))
    shape = list(a.shape) if shape is None else list(shape)
    if strides is None:
        strides, s = [], 1
        for d in reversed(shape):
            strides.insert(0, s)
            s *= d
    return _wrap(a._t.as_strided(shape, list(strides), int(offset)))


def slice(a, start_indices, axes, slice_size, **_):  # noqa: A001  (MLX name)
    a = _arr(a)
    starts = [int(v) for v in np.asarray(start_indices).reshape(-1)]
    idx = [builtins.slice(None)] * a.ndim
    for st, ax, sz in zip(starts, axes, slice_size):
        idx[int(ax) % a.ndim] = builtins.slice(st, st + int(sz))
    return _wrap(a._t[tuple(idx)])


def slice_update(a, update, start_indices, axes, **_):
    a = _arr(a)
    u = _arr(update)
    out = contiguous_copy(a) if not a._t.is_contiguous() else _wrap(a._t.clone())
    starts = [int(v) for v in np.asarray(start_indices).reshape(-1)]
    idx = [builtins.slice(None)] * a.ndim
    for st, ax in zip(starts, axes):
        ax = int(ax) % a.ndim
        idx[ax] = builtins.slice(st, st + u.shape[ax - (a.ndim - u.ndim)] if u.ndim == a.ndim else st + 1)
    _copy_into(out._t[tuple(idx)], broadcast_to(u, tuple(out._t[tuple(idx)].shape))._t)
    return out


def asarray(a, dtype=None, **_):
    return array(a, dtype)


def hadamard_transform(a, scale: float | None = None, **_):
    """x @ H_n (Sylvester Hadamard matrix of the last axis' power-of-two
    size) * scale, default scale 1/sqrt(n), on this backend's GEMM."""
    from ..ops import matmul

    a = _arr(a)
    n = a.shape[-1]
    if n & (n - 1):
        raise ValueError("hadamard_transform: the last axis must be a power of two")
    h = np.ones((1, 1), np.float32)
    while h.shape[0] < n:
        h = np.block([[h, h], [h, -h]])
    s = (1.0 / math.sqrt(n)) if scale is None else scale
    hd = array((h * s).astype(np.float32), a.dtype if a.dtype.kind == "f" else dt.float32)
    return matmul(a, hd)
