"""ORACLE -- test infrastructure only.

A CPU restatement of the MLX-CPU evaluation that phew's candidate path is
checked against.  Only ``tests/``, ``__graft_entry__.smoke()`` and
``bench.py``'s CPU-baseline leg (``cpu_baseline`` / ``--impl reference``)
may import it, and only as the checker or the timed CPU baseline -- never as
part of the product path.

Parity status
-------------
* Numerics: PARITY UNPINNED.  The reference evaluates through MLX 0.31.2 /
  mlx-metal 0.31.2 (phew ``uv.lock:399-400,434-435``), which is not
  installed here, and the reference's tests pin no numeric results at that
  boundary.  This module restates MLX's op semantics from the reference's
  call sites: op order from ``emit/codegen.py:94-476``, fused-kernel
  arithmetic from ``emit/msl_codegen.py:184-330`` (every node rounded to its
  dtype), ``FastRMSNorm`` eps default from ``ir/ops.py:156-161``, SDPA scale
  from ``rules/primitive_subst.py:457-472`` with the mask dropped
  (``:490-495``).
* Verdict logic (``oracle/verdict.py``): PINNED against the reference's own
  ``EquivalenceChecker._allclose``, ``TOLERANCES`` and bench ``compare`` /
  ``check_convergence`` via committed golden fixtures
  (``tests/golden/make_golden.py``).

Semantics restated here (MLX-CPU):
* elementwise ops compute in fp32 and round the result to the node dtype;
* Python scalars are weak (take the array's dtype; ``_TracedArray._binop``,
  ``ir/importer.py:171-186``, records them as Constants of that dtype);
* reductions, softmax, rms_norm and SDPA accumulate in float64 and round
  once to the output dtype; matmul accumulates in fp32 (BLAS sgemm);
* ``fast.rms_norm``: y = w * T(x * rsqrt(mean(x^2) + eps));
* ``fast.layer_norm``: y = T(w * T((x - mean) * rsqrt(var + eps)) + b);
* ``fast.rope``: fp32 angle position * scale * base^(-2i/dims), rotated
  pairs (i, i + dims/2) or, traditional, (2i, 2i+1).
"""

from __future__ import annotations

import math
import types
from typing import Any

import ml_dtypes
import numpy as np
from scipy import special as _sp

BF16 = np.dtype(ml_dtypes.bfloat16)

_NP = {
    "float32": np.dtype(np.float32),
    "float16": np.dtype(np.float16),
    "bfloat16": BF16,
    "int8": np.dtype(np.int8),
    "int16": np.dtype(np.int16),
    "int32": np.dtype(np.int32),
    "int64": np.dtype(np.int64),
    "uint8": np.dtype(np.uint8),
    "uint16": np.dtype(np.uint16),
    "uint32": np.dtype(np.uint32),
    "uint64": np.dtype(np.uint64),
    "bool": np.dtype(np.bool_),
}


class Dtype:
    def __init__(self, name: str) -> None:
        self.name = name
        self.np = _NP[name]
        self.size = self.np.itemsize
        self.kind = "f" if name in ("float32", "float16", "bfloat16") else (
            "b" if name == "bool" else ("u" if name.startswith("uint") else "i"))

    @property
    def value(self) -> str:
        return self.name

    def __repr__(self) -> str:
        return f"oracle.{self.name}"


float32, float16, bfloat16 = Dtype("float32"), Dtype("float16"), Dtype("bfloat16")
int8, int16, int32, int64 = Dtype("int8"), Dtype("int16"), Dtype("int32"), Dtype("int64")
uint8, uint16, uint32, uint64 = Dtype("uint8"), Dtype("uint16"), Dtype("uint32"), Dtype("uint64")
bool_ = Dtype("bool")
_BY_NAME = {d.name: d for d in (float32, float16, bfloat16, int8, int16, int32, int64, uint8,
                                uint16, uint32, uint64, bool_)}
_BY_NAME["bool_"] = bool_


def as_dtype(d: Any) -> Dtype:
    if isinstance(d, Dtype):
        return d
    v = getattr(d, "value", None) or getattr(d, "name", None)
    if isinstance(v, str) and v in _BY_NAME:
        return _BY_NAME[v]
    if isinstance(d, str):
        return _BY_NAME[d]
    nd = np.dtype(d)
    if nd == BF16:
        return bfloat16
    if nd == np.float64:
        return float32
    return _BY_NAME["bool" if nd == np.bool_ else nd.name]


def round_to(x: np.ndarray, d: Dtype) -> np.ndarray:
    """Round values (any float array) to dtype `d`, returned in dtype `d`."""
    if d.kind == "f":
        return np.asarray(x, dtype=np.float32).astype(d.np)
    return np.asarray(x).astype(d.np)


def f32(x: np.ndarray) -> np.ndarray:
    return np.asarray(x).astype(np.float32)


def _promote(a: Dtype, b: Dtype) -> Dtype:
    if a is b:
        return a
    if a.kind == "f" and b.kind == "f":
        if {a.name, b.name} == {"float16", "bfloat16"}:
            return float32
        rank = {"float16": 1, "bfloat16": 1, "float32": 2}
        return a if rank[a.name] >= rank[b.name] else b
    if a.kind == "f":
        return a
    if b.kind == "f":
        return b
    if a.kind == "b":
        return b
    if b.kind == "b":
        return a
    return a if a.size >= b.size else b


class array:
    """Host array with an MLX dtype; values stored in that dtype."""

    __array_priority__ = 100

    def __init__(self, val: Any, dtype: Any = None) -> None:
        if isinstance(val, array):
            v = val.v if dtype is None else round_to(f32(val.v) if val.dtype.kind == "f" else val.v, as_dtype(dtype))
            self.v = v
            self.dtype = val.dtype if dtype is None else as_dtype(dtype)
            return
        a = np.asarray(val)
        if dtype is None:
            if a.dtype == np.float64:
                d = float32
            elif a.dtype == np.int64 and not isinstance(val, np.ndarray):
                d = int32
            else:
                d = as_dtype(a.dtype)
        else:
            d = as_dtype(dtype)
        self.dtype = d
        self.v = round_to(a.astype(np.float64) if d.kind == "f" and a.dtype.kind != "V" and a.dtype != BF16 else a, d)

    @classmethod
    def wrap(cls, v: np.ndarray, d: Dtype) -> "array":
        a = object.__new__(cls)
        a.v = v
        a.dtype = d
        return a

    @property
    def shape(self):
        return tuple(self.v.shape)

    @property
    def size(self):
        return int(self.v.size)

    @property
    def ndim(self):
        return self.v.ndim

    def __array__(self, dtype=None, copy=None):
        out = self.v
        return out.astype(dtype) if dtype is not None else out

    def astype(self, d):
        return astype(self, d)

    @property
    def T(self):
        return transpose(self)

    def transpose(self, *axes):
        if len(axes) == 1 and isinstance(axes[0], (list, tuple)):
            axes = tuple(axes[0])
        return transpose(self, axes or None)

    def reshape(self, *shape):
        if len(shape) == 1 and isinstance(shape[0], (list, tuple)):
            shape = tuple(shape[0])
        return array.wrap(self.v.reshape(shape), self.dtype)

    def swapaxes(self, a, b):
        return array.wrap(np.swapaxes(self.v, a, b), self.dtype)

    def __getitem__(self, idx):
        return array.wrap(self.v[idx], self.dtype)

    def sum(self, axis=None, keepdims=False):
        return sum(self, axis, keepdims)

    def mean(self, axis=None, keepdims=False):
        return mean(self, axis, keepdims)

    def max(self, axis=None, keepdims=False):
        return max(self, axis, keepdims)

    def __add__(self, o):
        return _ew("add", self, o)

    def __radd__(self, o):
        return _ew("add", o, self)

    def __sub__(self, o):
        return _ew("sub", self, o)

    def __rsub__(self, o):
        return _ew("sub", o, self)

    def __mul__(self, o):
        return _ew("mul", self, o)

    def __rmul__(self, o):
        return _ew("mul", o, self)

    def __truediv__(self, o):
        return _ew("div", self, o)

    def __rtruediv__(self, o):
        return _ew("div", o, self)

    def __neg__(self):
        return _ew("negative", self)

    def __matmul__(self, o):
        return matmul(self, o)


# ---------------------------------------------------------------------------
# elementwise (fp32 compute, result rounded to the node dtype)
# ---------------------------------------------------------------------------


def _sigmoid(a):
    with np.errstate(over="ignore"):
        return np.float32(1.0) / (np.float32(1.0) + np.exp(-a))


def _maximum(a, b):
    return np.maximum(a, b)


def _remainder(a, b):
    return np.remainder(a, b)


FLOAT_OPS = {
    "add": lambda a, b: a + b,
    "sub": lambda a, b: a - b,
    "mul": lambda a, b: a * b,
    "div": lambda a, b: a / b,
    "negative": lambda a: -a,
    "abs": np.abs,
    "exp": np.exp,
    "log": np.log,
    "sqrt": np.sqrt,
    "rsqrt": lambda a: np.float32(1.0) / np.sqrt(a),
    "sigmoid": _sigmoid,
    "tanh": np.tanh,
    "relu": lambda a: np.maximum(a, np.float32(0.0)),
    "gelu": lambda a: (a * np.float32(0.5)) * (np.float32(1.0) + _sp.erf(a * np.float32(0.70710678118654752))).astype(np.float32),
    "silu": lambda a: a / (np.float32(1.0) + np.exp(-a)),
    "cos": np.cos,
    "sin": np.sin,
    "tan": np.tan,
    "arctan": np.arctan,
    "arcsin": np.arcsin,
    "arccos": np.arccos,
    "arctanh": np.arctanh,
    "arcsinh": np.arcsinh,
    "arccosh": np.arccosh,
    "cosh": np.cosh,
    "sinh": np.sinh,
    "degrees": lambda a: a * np.float32(57.295779513082320876),
    "radians": lambda a: a * np.float32(0.017453292519943295769),
    "square": lambda a: a * a,
    "maximum": _maximum,
    "minimum": np.minimum,
    "logaddexp": np.logaddexp,
    "ceil": np.ceil,
    "floor": np.floor,
    "round": np.rint,
    "sign": np.sign,
    "reciprocal": lambda a: np.float32(1.0) / a,
    "erf": lambda a: _sp.erf(a).astype(np.float32),
    "erfinv": lambda a: _sp.erfinv(a).astype(np.float32),
    "expm1": np.expm1,
    "log1p": np.log1p,
    "log2": np.log2,
    "log10": np.log10,
    "floor_divide": lambda a, b: np.floor(a / b),
    "remainder": _remainder,
    "power": np.power,
    "arctan2": np.arctan2,
}
ALIASES = {"multiply": "mul", "subtract": "sub", "divide": "div", "neg": "negative"}
COMPARE = {"eq": np.equal, "ne": np.not_equal, "gt": np.greater, "ge": np.greater_equal,
           "lt": np.less, "le": np.less_equal}


def _operand(x, d: Dtype):
    if isinstance(x, array):
        return x.v
    return round_to(np.asarray(x, dtype=np.float64 if d.kind == "f" else None), d)


def apply_op(op: str, args: list[np.ndarray], out: Dtype) -> np.ndarray:
    """One elementwise node: inputs already in their node dtypes."""
    op = ALIASES.get(op, op)
    if op in COMPARE:
        r = COMPARE[op](*[f32(a) if out.kind == "f" or a.dtype.kind == "f" else a for a in args])
        return round_to(r, out)
    if op == "where":
        return round_to(np.where(args[0].astype(bool), f32(args[1]), f32(args[2])), out)
    if op == "logical_not":
        return round_to(np.logical_not(args[0]), out)
    if op in ("logical_and", "logical_or"):
        f = np.logical_and if op == "logical_and" else np.logical_or
        return round_to(f(args[0], args[1]), out)
    if out.kind != "f":
        f = {"add": np.add, "sub": np.subtract, "mul": np.multiply, "negative": np.negative,
             "abs": np.abs, "maximum": np.maximum, "minimum": np.minimum,
             "floor_divide": np.floor_divide, "remainder": np.remainder, "square": np.square,
             "sign": np.sign}[op]
        return f(*[a.astype(out.np) for a in args]).astype(out.np)
    with np.errstate(all="ignore"):
        r = FLOAT_OPS[op](*[f32(a) for a in args])
    return round_to(np.asarray(r, dtype=np.float32), out)


def _ew(op: str, *operands) -> array:
    arrays = [x for x in operands if isinstance(x, array)]
    res = arrays[0].dtype
    for a in arrays[1:]:
        res = _promote(res, a.dtype)
    for x in operands:
        if not isinstance(x, array) and isinstance(x, float) and res.kind != "f":
            res = float32
    args = []
    for x in operands:
        if isinstance(x, array):
            args.append(x.v if x.dtype is res else round_to(f32(x.v) if x.dtype.kind == "f" else x.v, res))
        else:
            args.append(_operand(x, res))
    return array.wrap(apply_op(op, args, res), res)


def _unary_fn(op):
    return lambda x, *_, **__: _ew(op, x)


for _op in ("exp", "log", "sqrt", "rsqrt", "sigmoid", "tanh", "abs", "negative", "square", "sin",
            "cos", "erf", "erfinv", "expm1", "log1p", "log2", "log10", "ceil", "floor", "round",
            "sign", "reciprocal", "arctan", "arcsin", "arccos", "sinh", "cosh", "relu", "gelu",
            "silu"):
    globals()[_op] = _unary_fn(_op)

maximum = lambda a, b: _ew("maximum", a, b)  # noqa: E731
minimum = lambda a, b: _ew("minimum", a, b)  # noqa: E731
power = lambda a, b: _ew("power", a, b)  # noqa: E731
add = lambda a, b: _ew("add", a, b)  # noqa: E731
multiply = lambda a, b: _ew("mul", a, b)  # noqa: E731
subtract = lambda a, b: _ew("sub", a, b)  # noqa: E731
divide = lambda a, b: _ew("div", a, b)  # noqa: E731


def astype(a: array, d) -> array:
    d = as_dtype(d)
    if a.dtype is d:
        return a
    if d.kind == "f":
        return array.wrap(round_to(f32(a.v), d), d)
    if a.dtype.kind == "f":
        return array.wrap(np.trunc(f32(a.v)).astype(d.np), d)
    return array.wrap(a.v.astype(d.np), d)


def where(c, a, b):
    cv = c.v if isinstance(c, array) else np.asarray(c)
    res = a.dtype if isinstance(a, array) else b.dtype
    av = _operand(a, res) if not isinstance(a, array) else astype(a, res).v
    bv = _operand(b, res) if not isinstance(b, array) else astype(b, res).v
    return array.wrap(round_to(np.where(cv.astype(bool), f32(av), f32(bv)), res), res)


# ---------------------------------------------------------------------------
# reductions, softmax, matmul, fast.*
# ---------------------------------------------------------------------------


def _axes(a: array, axis):
    if axis is None:
        return tuple(range(a.ndim))
    if isinstance(axis, (list, tuple)):
        return tuple(int(x) % a.ndim for x in axis)
    return (int(axis) % a.ndim,)


def _reduce(fn, a: array, axis, keepdims) -> array:
    ax = _axes(a, axis)
    with np.errstate(all="ignore"):
        r = fn(a.v.astype(np.float64), axis=ax, keepdims=keepdims)
    return array.wrap(round_to(r, a.dtype), a.dtype)


def sum(a, axis=None, keepdims=False, **_):  # noqa: A001
    return _reduce(np.sum, a, axis, keepdims)


def mean(a, axis=None, keepdims=False, **_):
    return _reduce(np.mean, a, axis, keepdims)


def max(a, axis=None, keepdims=False, **_):  # noqa: A001
    return _reduce(np.max, a, axis, keepdims)


def min(a, axis=None, keepdims=False, **_):  # noqa: A001
    return _reduce(np.min, a, axis, keepdims)


def var(a, axis=None, keepdims=False, ddof=0, **_):
    ax = _axes(a, axis)
    x = a.v.astype(np.float64)
    n = int(np.prod([a.shape[i] for i in ax])) if ax else 1
    with np.errstate(all="ignore"):
        d = x - x.mean(axis=ax, keepdims=True)
        r = (d * d).sum(axis=ax, keepdims=keepdims) / (n - ddof)
    return array.wrap(round_to(r, a.dtype), a.dtype)


def std(a, axis=None, keepdims=False, ddof=0, **_):
    return _ew("sqrt", var(a, axis, keepdims, ddof))


def logsumexp(a, axis=None, keepdims=False, **_):
    x = a.v.astype(np.float64)
    ax = _axes(a, axis)
    with np.errstate(all="ignore"):
        m = np.max(x, axis=ax, keepdims=True)
        m = np.where(np.isinf(m), 0.0, m)
        r = np.log(np.sum(np.exp(x - m), axis=ax, keepdims=True)) + m
    if not keepdims:
        r = np.squeeze(r, axis=ax)
    return array.wrap(round_to(r, a.dtype), a.dtype)


def _pred(fn):
    return lambda a, *_, **__: array.wrap(fn(f32(a.v)), as_dtype("bool"))


isnan = _pred(np.isnan)
isinf = _pred(np.isinf)
isfinite = _pred(np.isfinite)
isposinf = _pred(np.isposinf)
isneginf = _pred(np.isneginf)


def clip(a, a_min=None, a_max=None, **_):
    out = a
    if a_min is not None:
        out = _ew("maximum", out, a_min)
    if a_max is not None:
        out = _ew("minimum", out, a_max)
    return out


def all(a, axis=None, keepdims=False, **_):  # noqa: A001
    return array.wrap(np.all(a.v != 0, axis=_axes(a, axis), keepdims=keepdims), as_dtype("bool"))


def any(a, axis=None, keepdims=False, **_):  # noqa: A001
    return array.wrap(np.any(a.v != 0, axis=_axes(a, axis), keepdims=keepdims), as_dtype("bool"))


def concatenate(arrays, axis=0, **_):
    res = arrays[0].dtype
    for x in arrays[1:]:
        res = _promote(res, x.dtype)
    if axis is None:
        return array.wrap(np.concatenate([astype(x, res).v.reshape(-1) for x in arrays]), res)
    return array.wrap(np.concatenate([astype(x, res).v for x in arrays], axis=axis), res)


concat = concatenate


def stack(arrays, axis=0, **_):
    return array.wrap(np.stack([x.v for x in arrays], axis=axis), arrays[0].dtype)


def split(a, indices_or_sections, axis=0, **_):
    return [array.wrap(p, a.dtype) for p in np.split(a.v, indices_or_sections, axis=axis)]


def pad(a, pad_width, mode="constant", constant_values=0, **_):
    if isinstance(pad_width, int):
        pw = pad_width
    elif len(pad_width) and isinstance(pad_width[0], int):
        pw = [tuple(pad_width)] * a.ndim if len(pad_width) == 2 else [(p, p) for p in pad_width]
    else:
        pw = [tuple(p) for p in pad_width]
        if len(pw) == 1:
            pw = pw * a.ndim
    return array.wrap(np.pad(a.v, pw, constant_values=constant_values), a.dtype)


def tile(a, reps, **_):
    return array.wrap(np.tile(a.v, reps), a.dtype)


def repeat(a, repeats, axis=None, **_):
    return array.wrap(np.repeat(a.v, repeats, axis=axis), a.dtype)


def roll(a, shift, axis=None, **_):
    return array.wrap(np.roll(a.v, shift, axis=axis), a.dtype)


def tril(x, k=0, **_):
    return array.wrap(np.tril(x.v, k), x.dtype)


def triu(x, k=0, **_):
    return array.wrap(np.triu(x.v, k), x.dtype)


def cumsum(a, axis=None, reverse=False, inclusive=True, **_):
    x = a.v.reshape(-1) if axis is None else a.v
    ax = 0 if axis is None else axis
    if reverse:
        x = np.flip(x, ax)
    r = np.cumsum(x.astype(np.float64) if a.dtype.kind == "f" else x, axis=ax)
    if not inclusive:
        r = np.roll(r, 1, ax)
        idx = [np.s_[:]] * r.ndim
        idx[ax] = 0
        r[tuple(idx)] = 0
    if reverse:
        r = np.flip(r, ax)
    return array.wrap(round_to(r, a.dtype) if a.dtype.kind == "f" else r.astype(a.dtype.np), a.dtype)


def sort(a, axis=-1, **_):
    return array.wrap(np.sort(a.v.reshape(-1) if axis is None else a.v, axis=-1 if axis is None else axis,
                              kind="stable"), a.dtype)


def argsort(a, axis=-1, **_):
    return array.wrap(np.argsort(a.v.reshape(-1) if axis is None else a.v, axis=-1 if axis is None else axis,
                                 kind="stable").astype(np.int32), as_dtype("int32"))


def topk(a, k, axis=-1, **_):
    s = np.sort(a.v, axis=axis)
    return array.wrap(np.take(s, np.arange(s.shape[axis] - k, s.shape[axis]), axis=axis), a.dtype)


def argmax(a, axis=None, keepdims=False, **_):
    r = np.argmax(a.v, axis=axis, keepdims=keepdims) if axis is not None else np.argmax(a.v)
    return array.wrap(np.asarray(r).astype(np.uint32), as_dtype("uint32"))


def argmin(a, axis=None, keepdims=False, **_):
    r = np.argmin(a.v, axis=axis, keepdims=keepdims) if axis is not None else np.argmin(a.v)
    return array.wrap(np.asarray(r).astype(np.uint32), as_dtype("uint32"))


def take_along_axis(a, indices, axis=None, **_):
    if axis is None:
        return array.wrap(np.take_along_axis(a.v.reshape(-1), indices.v.reshape(-1).astype(np.int64), 0), a.dtype)
    return array.wrap(np.take_along_axis(a.v, indices.v.astype(np.int64), axis), a.dtype)


def take(a, indices, axis=None, **_):
    idx = indices.v if isinstance(indices, array) else np.asarray(indices)
    return array.wrap(np.take(a.v, idx.astype(np.int64), axis=axis), a.dtype)


def moveaxis(a, source, destination, **_):
    return array.wrap(np.moveaxis(a.v, source, destination), a.dtype)


def flatten(a, start_axis=0, end_axis=-1, **_):
    if a.ndim == 0:
        return reshape(a, (1,))
    s = start_axis % a.ndim
    e = end_axis % a.ndim
    shape = list(a.shape[:s]) + [int(np.prod(a.shape[s:e + 1]))] + list(a.shape[e + 1:])
    return reshape(a, shape)


def bitwise_and(a, b, **_):
    return array.wrap(np.bitwise_and(a.v, b.v if isinstance(b, array) else b), a.dtype)


def bitwise_or(a, b, **_):
    return array.wrap(np.bitwise_or(a.v, b.v if isinstance(b, array) else b), a.dtype)


def bitwise_xor(a, b, **_):
    return array.wrap(np.bitwise_xor(a.v, b.v if isinstance(b, array) else b), a.dtype)


def left_shift(a, b, **_):
    return array.wrap(np.left_shift(a.v, b.v if isinstance(b, array) else b), a.dtype)


def right_shift(a, b, **_):
    return array.wrap(np.right_shift(a.v, b.v if isinstance(b, array) else b), a.dtype)


def dequantize(w, scales, biases, group_size=64, bits=4, **_):
    """Affine group-wise codes, 32/bits per uint32 along the last axis (code j
    of a word in bits [j*bits, (j+1)*bits)) -> T(fma(scale, q, bias))."""
    per = 32 // bits
    words = np.asarray(w.v).astype(np.uint64)
    shifts = (np.arange(per, dtype=np.uint64) * np.uint64(bits))
    q = ((words[..., None] >> shifts) & np.uint64((1 << bits) - 1)).reshape(*words.shape[:-1], -1)
    s = np.repeat(f32(scales.v).astype(np.float64), group_size, axis=-1)
    b = np.repeat(f32(biases.v).astype(np.float64), group_size, axis=-1)
    r = (s * q.astype(np.float64) + b).astype(np.float32)
    return array.wrap(round_to(r, scales.dtype), scales.dtype)


def quantized_matmul(x, w, scales=None, biases=None, transpose=True, group_size=64, bits=4, **_):
    if scales is None or biases is None:
        raise TypeError("quantized_matmul: scales and biases are required for affine quantization")
    wd = dequantize(w, scales, biases, group_size, bits)
    return matmul(astype(x, wd.dtype), swapaxes(wd, -1, -2) if transpose else wd)


def _softmax64(x: np.ndarray, axis: int) -> np.ndarray:
    with np.errstate(all="ignore"):
        m = np.max(x, axis=axis, keepdims=True)
        e = np.exp(x - m)
        return e / np.sum(e, axis=axis, keepdims=True)


def softmax(a, axis=-1, **_):
    if isinstance(axis, (list, tuple)):
        axis = axis[0]
    return array.wrap(round_to(_softmax64(a.v.astype(np.float64), int(axis)), a.dtype), a.dtype)


def matmul(a, b):
    res = _promote(a.dtype, b.dtype)
    r = np.matmul(f32(a.v), f32(b.v))
    return array.wrap(round_to(r, res), res)


def transpose(a, axes=None):
    return array.wrap(np.transpose(a.v, axes), a.dtype)


def swapaxes(a, x, y):
    return array.wrap(np.swapaxes(a.v, x, y), a.dtype)


def reshape(a, shape):
    return array.wrap(a.v.reshape(shape), a.dtype)


def zeros_like(a):
    return array.wrap(np.zeros(a.shape, a.dtype.np), a.dtype)


def zeros(shape, dtype=float32):
    d = as_dtype(dtype)
    return array.wrap(np.zeros(shape, d.np), d)


def ones(shape, dtype=float32):
    d = as_dtype(dtype)
    return array.wrap(np.ones(shape, d.np), d)


def eval(*_):  # noqa: A001
    return None


def synchronize(*_):
    return None


def compile(fn=None, **_):  # noqa: A001
    return fn if fn is not None else (lambda f: f)


def rms_norm(x: array, weight: array | None = None, eps: float = 1e-5) -> array:
    """fast.rms_norm: fp32 mean of squares, then y = w * T(x * r).  The
    weight must be 1-D over the last axis, as MLX requires."""
    cols = x.shape[-1]
    if weight is not None and tuple(weight.shape) != (cols,):
        raise ValueError(f"rms_norm: weight shape {tuple(weight.shape)} != ({cols},)")
    xv = f32(x.v)
    ms = np.float32(np.mean(xv.astype(np.float64) ** 2, axis=-1, keepdims=True))
    r = (np.float32(1.0) / np.sqrt(ms + np.float32(eps))).astype(np.float32)
    n = round_to(xv * r, x.dtype)
    if weight is None:
        return array.wrap(n, x.dtype)
    return array.wrap(round_to(f32(weight.v) * f32(n), x.dtype), x.dtype)


def layer_norm(x: array, weight: array | None = None, bias: array | None = None,
               eps: float = 1e-5) -> array:
    """fast.layer_norm (``ir/ops.py:165-168``): float64 mean and biased
    variance of the row, n = T((x - mean) * rsqrt(var + eps)), then
    y = T(fp32(w * n) + b) with weight / bias omitted when None."""
    cols = x.shape[-1]
    for p, nm in ((weight, "weight"), (bias, "bias")):
        if p is not None and tuple(p.shape) != (cols,):
            raise ValueError(f"layer_norm: {nm} shape {tuple(p.shape)} != ({cols},)")
    xv = f32(x.v).astype(np.float64)
    mean = xv.mean(axis=-1, keepdims=True)
    var = ((xv - mean) ** 2).mean(axis=-1, keepdims=True)
    n = f32(round_to((xv - mean) / np.sqrt(var + eps), x.dtype))
    if weight is not None:
        n = (n * f32(weight.v)).astype(np.float32)
    if bias is not None:
        n = (n + f32(bias.v)).astype(np.float32)
    return array.wrap(round_to(n, x.dtype), x.dtype)


def rope(x: array, dims: int, *, traditional: bool = False, base: float = 10000.0,
         scale: float = 1.0, offset: int = 0) -> array:
    """fast.rope (``ir/ops.py:172-179``): positions offset + l along the
    second-to-last axis; pair i of the first `dims` features, (i, i + dims/2)
    or (2i, 2i+1) when traditional, rotates by the fp32 angle
    fp32(fp32(pos * scale) * fp32(base^(-2i/dims))); each product and sum
    in fp32; the rest of the features are copied."""
    xv = f32(x.v)
    shp = xv.shape
    D = shp[-1]
    L = shp[-2] if len(shp) >= 2 else 1
    half = dims // 2
    out = xv.copy()
    if half:
        inv = np.power(np.float64(base), -2.0 * np.arange(half) / dims).astype(np.float32)
        pos = (np.float32(offset) + np.arange(L, dtype=np.float32)).astype(np.float32)
        a = ((pos * np.float32(scale)).astype(np.float32)[:, None] * inv[None, :]).astype(np.float32)
        c = np.cos(a.astype(np.float64)).astype(np.float32)
        sn = np.sin(a.astype(np.float64)).astype(np.float32)
        if traditional:
            iu, iv = np.arange(half) * 2, np.arange(half) * 2 + 1
        else:
            iu, iv = np.arange(half), np.arange(half) + half
        u, v = xv[..., iu], xv[..., iv]
        out[..., iu] = ((u * c).astype(np.float32) - (v * sn).astype(np.float32)).astype(np.float32)
        out[..., iv] = ((u * sn).astype(np.float32) + (v * c).astype(np.float32)).astype(np.float32)
    _ = D
    return array.wrap(round_to(out, x.dtype), x.dtype)


def sdpa(q: array, k: array, v: array, scale: float, mask: Any = None) -> array:
    """softmax(q k^T * scale [+ mask]) v, fp32 matmuls, float64 softmax."""
    s = np.matmul(f32(q.v), np.swapaxes(f32(k.v), -1, -2)) * np.float32(scale)
    s = s.astype(np.float64)
    if isinstance(mask, str) and mask == "causal":
        L, S = s.shape[-2], s.shape[-1]
        s = np.where(np.tril(np.ones((L, S), dtype=bool), k=S - L), s, -np.inf)
    elif mask is not None:
        s = s + f32(mask.v if isinstance(mask, array) else mask)
    p = _softmax64(s, -1).astype(np.float32)
    o = np.matmul(p, f32(v.v))
    return array.wrap(round_to(o, q.dtype), q.dtype)


# Fused kernels appear in emitted sources as CUDA bodies; the oracle evaluates
# the chain each body was emitted from (registered by sha1 of the body).
CUDA_CHAINS: dict[str, dict] = {}


class _ChainKernel:
    def __init__(self, source: str) -> None:
        import hashlib

        from phew_b200.graph import NodeSpec

        key = hashlib.sha1(source.encode()).hexdigest()
        if key not in CUDA_CHAINS:
            raise KeyError("oracle: no chain registered for this fused kernel body")
        rec = CUDA_CHAINS[key]
        self.nodes = [NodeSpec.from_json(d) for d in rec["nodes"]]
        self.ins = [NodeSpec.from_json(d) for d in rec["ext_inputs"]]
        self.outs = [NodeSpec.from_json(d) for d in rec["ext_outputs"]]

    def __call__(self, inputs, output_shapes, output_dtypes, grid=None, threadgroup=None,
                 template=None, **_):
        vals = [x.v if isinstance(x, array) else np.asarray(x) for x in inputs]
        outs = []
        for spec, shp, dt in zip(self.outs, output_shapes, output_dtypes):
            spec.shape = tuple(shp)
        res = eval_chain(self.nodes, self.ins, self.outs, vals)
        for r, shp, dt in zip(res, output_shapes, output_dtypes):
            d = as_dtype(dt)
            outs.append(array.wrap(r.reshape(shp).astype(d.np), d))
        return outs


def cuda_kernel(name, input_names, output_names, source, header="", **_):
    return _ChainKernel(source)


fast = types.SimpleNamespace(
    rms_norm=rms_norm,
    layer_norm=lambda x, weight=None, bias=None, eps=1e-5, **_: layer_norm(x, weight, bias, eps),
    rope=lambda x, dims, **kw: rope(x, dims, **kw),
    scaled_dot_product_attention=lambda q, k, v, *, scale=1.0, mask=None, **_: sdpa(q, k, v, scale, mask),
    cuda_kernel=cuda_kernel,
)


def elementwise_threads(n: int) -> int:
    """Launch size of emitted elementwise kernels (unused on the CPU)."""
    return int(n)


# ---------------------------------------------------------------------------
# fused-chain evaluation (node by node, each rounded to its dtype)
# ---------------------------------------------------------------------------


def _kind(n) -> str:
    return getattr(n, "kind", None) or type(n).__name__


def _dname(d) -> str:
    v = getattr(d, "value", None)
    if isinstance(v, str):
        d = v
    d = str(d)
    return "bool" if d == "bool_" else d


def eval_chain(nodes, ext_inputs, ext_outputs, values: list[np.ndarray]) -> list[np.ndarray]:
    """Evaluate an Elementwise/Cast/Constant chain the way the MSL kernel and
    MLX's op-by-op evaluation do (``msl_codegen.py:184-330``)."""
    env: dict[int, np.ndarray] = {}
    out_shape = tuple(ext_outputs[0].shape)
    for node, v in zip(ext_inputs, values):
        env[node.id] = np.asarray(v)
    for node in nodes:
        kind = _kind(node)
        d = as_dtype(_dname(node.dtype))
        if kind == "Constant":
            env[node.id] = round_to(np.asarray(float(np.float32(node.value)) if d.kind == "f" else node.value), d)
        elif kind == "Cast":
            t = as_dtype(_dname(getattr(node, "target_dtype", node.dtype)))
            env[node.id] = astype(array.wrap(env[node.inputs[0]], as_dtype(env[node.inputs[0]].dtype)), t).v
        else:
            args = [env[i] for i in node.inputs]
            env[node.id] = apply_op(node.op, args, d)
    return [np.broadcast_to(env[o.id], out_shape).copy() for o in ext_outputs]


def to_float(x) -> np.ndarray:
    """Values of an oracle/device/numpy array as float32 numpy."""
    v = x.v if isinstance(x, array) else np.asarray(x)
    return v.astype(np.float32)


__all__ = [n for n in dir() if not n.startswith("_")]
