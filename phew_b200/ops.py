"""Hand-written primitive ops on ``phew_b200.mx`` arrays.

Each function validates shapes on the host and calls one C-ABI entry point
of ``libphew_b200.so`` on the current stream.
"""

from __future__ import annotations

import ctypes

from . import _native
from .mx.core import _stream, array, asarray_device, empty


def rms_norm(x, weight=None, eps: float = 1e-5) -> array:
    """``mx.fast.rms_norm(x, weight, eps)`` over the last axis.

    y = weight * cast(x * rsqrt(mean(x^2) + eps)); weight None -> no scaling.
    Node FastRMSNorm (phew ``ir/ops.py:156-161``), matched by
    ``rules/primitive_subst.py:63-145``, emitted at ``emit/codegen.py:401-404``.
    """
    x = asarray_device(x)
    if x.dtype.code is None:
        raise TypeError(f"rms_norm: unsupported dtype {x.dtype.name}")
    cols = x.shape[-1]
    rows = x.size // max(cols, 1)
    wptr = None
    if weight is not None:
        w = asarray_device(weight)
        if w.dtype is not x.dtype:
            w = w.astype(x.dtype)
        if w.shape != (cols,):
            raise ValueError(f"rms_norm: weight shape {w.shape} != ({cols},)")
        wptr = ctypes.c_void_p(w._t.data_ptr())
    out = empty(x.shape, x.dtype)
    if x.size:
        _native.call(
            "phew_rms_norm", ctypes.c_void_p(x._t.data_ptr()), wptr,
            ctypes.c_void_p(out._t.data_ptr()), rows, cols, ctypes.c_float(eps), x.dtype.code,
            _stream(),
        )
    return out


def matmul(a, b) -> array:
    raise NotImplementedError("matmul: the tcgen05 GEMM is not built yet")


def scaled_dot_product_attention(q, k, v, *, scale=1.0, mask=None) -> array:
    raise NotImplementedError("scaled_dot_product_attention: the tcgen05 kernel is not built yet")
