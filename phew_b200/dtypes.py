"""Array dtypes of the ``phew_b200.mx`` namespace.

Each dtype object mirrors an ``mlx.core`` dtype (``mx.float16`` ...): it is
hashable, has ``.size`` (bytes) and a ``.name`` equal to the value of the
matching ``phew.ir.dtype.Dtype`` member (``ir/dtype.py:6-20``), so phew's
``Dtype(...)`` lookups and ``to_mlx()`` names line up.
"""

from __future__ import annotations

import numpy as np
import torch

try:
    import ml_dtypes

    _NP_BF16 = np.dtype(ml_dtypes.bfloat16)
except ImportError:  # pragma: no cover
    _NP_BF16 = None


class Dtype:
    __slots__ = ("name", "size", "torch", "kind", "code", "np")

    def __init__(self, name: str, size: int, torch_dtype, kind: str, code: int | None, np_dtype):
        self.name = name
        self.size = size
        self.torch = torch_dtype
        self.kind = kind  # "f" float, "i" signed int, "u" unsigned int, "b" bool
        self.code = code  # C-ABI dtype code for the hand-written kernels
        self.np = np_dtype

    @property
    def value(self) -> str:  # same spelling as phew.ir.dtype.Dtype.value
        return self.name

    def __repr__(self) -> str:
        return f"phew_b200.mx.{self.name if self.name != 'bool' else 'bool_'}"

    def __reduce__(self):
        return (from_name, (self.name,))


float32 = Dtype("float32", 4, torch.float32, "f", 0, np.dtype(np.float32))
float16 = Dtype("float16", 2, torch.float16, "f", 1, np.dtype(np.float16))
bfloat16 = Dtype("bfloat16", 2, torch.bfloat16, "f", 2, _NP_BF16)
int8 = Dtype("int8", 1, torch.int8, "i", None, np.dtype(np.int8))
int16 = Dtype("int16", 2, torch.int16, "i", None, np.dtype(np.int16))
int32 = Dtype("int32", 4, torch.int32, "i", None, np.dtype(np.int32))
int64 = Dtype("int64", 8, torch.int64, "i", None, np.dtype(np.int64))
uint8 = Dtype("uint8", 1, torch.uint8, "u", None, np.dtype(np.uint8))
uint16 = Dtype("uint16", 2, torch.uint16, "u", None, np.dtype(np.uint16))
uint32 = Dtype("uint32", 4, torch.uint32, "u", None, np.dtype(np.uint32))
uint64 = Dtype("uint64", 8, torch.uint64, "u", None, np.dtype(np.uint64))
bool_ = Dtype("bool", 1, torch.bool, "b", None, np.dtype(np.bool_))

# Named for mlx.core compatibility (phew's Dtype.from_mlx table lists them,
# ir/dtype.py:70-88); arrays of these types are not supported on the GPU.
float64 = Dtype("float64", 8, torch.float64, "f", None, np.dtype(np.float64))
complex64 = Dtype("complex64", 8, torch.complex64, "c", None, np.dtype(np.complex64))

ALL = (float32, float16, bfloat16, int8, int16, int32, int64, uint8, uint16, uint32, uint64, bool_)
_BY_NAME = {d.name: d for d in ALL}
_BY_NAME["bool_"] = bool_
_BY_TORCH = {d.torch: d for d in ALL}


def from_name(name: str) -> Dtype:
    return _BY_NAME[name]


def from_any(d) -> Dtype:
    """Accept our Dtype, phew's Dtype enum, a numpy/torch dtype or a name."""
    if isinstance(d, Dtype):
        return d
    if isinstance(d, torch.dtype):
        return _BY_TORCH[d]
    v = getattr(d, "value", None)
    if isinstance(v, str) and v in _BY_NAME:
        return _BY_NAME[v]
    if isinstance(d, str):
        return _BY_NAME[d]
    nd = np.dtype(d)
    if _NP_BF16 is not None and nd == _NP_BF16:
        return bfloat16
    if nd == np.float64:
        raise TypeError("float64 arrays are not supported on the GPU (as in MLX)")
    return _BY_NAME["bool" if nd == np.bool_ else nd.name]


_FLOAT_RANK = {"float16": 1, "bfloat16": 1, "float32": 2}


def promote(a: Dtype, b: Dtype) -> Dtype:
    """Result dtype of a binary op on two arrays (MLX promotion rules)."""
    if a is b:
        return a
    if a.kind == "f" and b.kind == "f":
        if {a.name, b.name} == {"float16", "bfloat16"}:
            return float32
        return a if _FLOAT_RANK[a.name] >= _FLOAT_RANK[b.name] else b
    if a.kind == "f":
        return a
    if b.kind == "f":
        return b
    if a.kind == "b":
        return b
    if b.kind == "b":
        return a
    if a.kind == b.kind:
        return a if a.size >= b.size else b
    # signed/unsigned mix: widen to a signed type that holds both
    size = max(a.size, b.size) * (2 if (a.kind == "u" and a.size >= b.size) or (b.kind == "u" and b.size >= a.size) else 1)
    return {1: int8, 2: int16, 4: int32}.get(size, int64)


def scalar_dtype(value, other: Dtype) -> Dtype:
    """Dtype of (array `other`) op (Python scalar `value`): the scalar is weak."""
    if isinstance(value, bool):
        return other
    if isinstance(value, int):
        return other
    if isinstance(value, float):
        return other if other.kind == "f" else float32
    raise TypeError(f"unsupported scalar {value!r}")
