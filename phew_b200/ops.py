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


_error_flags: dict[int, object] = {}


def error_flag():
    """Device int that bounded in-kernel waits set on timeout (0 = clean)."""
    import torch

    from .mx.core import device

    dev = device()
    f = _error_flags.get(dev.index)
    if f is None:
        f = torch.zeros(1, dtype=torch.int32, device=dev)
        _error_flags[dev.index] = f
    return f


def check_device_errors() -> None:
    """Raise if any kernel reported a timed-out wait (synchronises)."""
    f = error_flag()
    code = int(f.item())
    if code:
        f.zero_()
        raise _native.PhewError(code, "a device-side wait timed out (pipeline stalled)")


def _collapse_batch(t, batch_shape) -> int | None:
    """Single element stride over the flattened batch dims, or None."""
    nb = len(batch_shape)
    if nb == 0:
        return 0
    strides = [t.stride(i) for i in range(nb)]
    shape = list(batch_shape)
    live = [(s, n) for s, n in zip(strides, shape) if n != 1]
    if not live:
        return 0
    if all(s == 0 for s, _ in live):
        return 0
    for i in range(len(live) - 1):
        if live[i][0] != live[i + 1][0] * live[i + 1][1]:
            return None
    return live[-1][0]


def matmul(a, b, *, row_scale: bool = False, eps: float = 1e-5) -> array:
    """``a @ b`` with MLX semantics (batched, broadcast batch dims, 1-D
    operands promoted), on the tcgen05 GEMM.

    ``row_scale=True`` returns ``(a @ b) * rsqrt(mean(a*a, -1) + eps)`` in one
    kernel (the normed matmul of ``rules/primitive_subst.py:156-240``).
    """
    from . import dtypes as dt
    from .mx.core import _broadcast_shapes, astype, contiguous_copy, reshape

    a = asarray_device(a, contiguous=False)
    b = asarray_device(b, contiguous=False)
    squeeze_a = a.ndim == 1
    squeeze_b = b.ndim == 1
    if squeeze_a:
        a = reshape(a, (1, a.shape[0]))
    if squeeze_b:
        b = reshape(b, (b.shape[0], 1))
    res = dt.promote(a.dtype, b.dtype)
    if res.code is None:
        raise TypeError(f"matmul: unsupported dtype {res.name}")
    if a.dtype is not res:
        a = astype(a, res)
    if b.dtype is not res:
        b = astype(b, res)
    M, K = a.shape[-2:]
    K2, N = b.shape[-2:]
    if K != K2:
        raise ValueError(f"matmul: inner dimensions differ ({a.shape} @ {b.shape})")
    batch_shape = _broadcast_shapes(a.shape[:-2], b.shape[:-2])
    nbatch = 1
    for s in batch_shape:
        nbatch *= s

    ta = a._t.expand(*batch_shape, M, K)
    if ta.stride(-1) != 1 and K > 1 or _collapse_batch(ta, batch_shape) is None:
        ta = contiguous_copy(array._wrap(ta))._t
    lda = ta.stride(-2) if M > 1 else K
    sa = _collapse_batch(ta, batch_shape)

    tb = b._t.expand(*batch_shape, K, N)
    layout = None
    if (tb.stride(-1) == 1 or N == 1) and (K == 1 or tb.stride(-2) >= N):
        layout, ldb = 0, (tb.stride(-2) if K > 1 else N)
    elif (tb.stride(-2) == 1 or K == 1) and (N == 1 or tb.stride(-1) >= K):
        layout, ldb = 1, (tb.stride(-1) if N > 1 else K)
    if layout is None or _collapse_batch(tb, batch_shape) is None:
        tb = contiguous_copy(array._wrap(tb))._t
        layout, ldb = 0, N
    sb = _collapse_batch(tb, batch_shape)

    out = empty(tuple(batch_shape) + (M, N), res)
    if out.size:
        _native.call(
            "phew_gemm",
            ctypes.c_void_p(ta.data_ptr()), ctypes.c_void_p(tb.data_ptr()),
            ctypes.c_void_p(out._t.data_ptr()),
            M, N, K, nbatch, lda, ldb, N, sa, sb, M * N if nbatch > 1 else 0,
            layout, res.code, res.code, int(row_scale), ctypes.c_float(eps),
            ctypes.c_void_p(error_flag().data_ptr()), _stream(),
        )
    if squeeze_a:
        out = reshape(out, out.shape[:-2] + (N,))
    if squeeze_b:
        out = reshape(out, out.shape[:-1])
    return out


def normed_matmul(x, w, eps: float = 1e-5) -> array:
    """``(x @ w) * rsqrt(mean(x*x, -1) + eps)`` fused into the GEMM."""
    return matmul(x, w, row_scale=True, eps=eps)


_mask_cache: dict[tuple, array] = {}


def causal_mask(L: int, S: int, dtype) -> array:
    """Additive causal mask (0 on and below the diagonal, -inf above),
    aligned bottom-right when S > L, cached per shape and dtype."""
    import numpy as np

    from .mx.core import array as _array

    key = (L, S, dtype.name)
    m = _mask_cache.get(key)
    if m is None:
        host = np.zeros((L, S), np.float32)
        host[np.triu_indices(L, S - L + 1, S)] = -np.inf
        m = _array(host, dtype)
        _mask_cache[key] = m
    return m


def scaled_dot_product_attention(q, k, v, *, scale=1.0, mask=None) -> array:
    """``mx.fast.scaled_dot_product_attention(q, k, v, scale=, mask=)``.

    q, k, v: [B, H, L, D].  ``mask`` None (no mask), ``"causal"`` or an
    additive array broadcastable to [B, H, L, S].  The fused tcgen05 kernel
    runs for D = 128, L = S multiple of 128, bf16/fp16, equal head counts,
    scale > 0 and mask None / "causal"; any other case is composed from this backend's GEMM
    and softmax kernels (scores materialised in HBM).
    """
    from .mx.core import astype, softmax, swapaxes

    q = asarray_device(q)
    k = asarray_device(k)
    v = asarray_device(v)
    causal = isinstance(mask, str) and mask == "causal"
    if isinstance(mask, str) and not causal:
        raise ValueError(f"unknown mask mode {mask!r}")
    fast_ok = (
        q.ndim == 4 and q.shape == k.shape == v.shape and q.dtype is k.dtype is v.dtype
        and q.dtype.name in ("bfloat16", "float16") and q.shape[-1] == 128
        and q.shape[-2] % 128 == 0 and (mask is None or causal) and float(scale) > 0.0
    )
    if fast_ok:
        B, H, L, D = q.shape
        out = empty(q.shape, q.dtype)
        _native.call(
            "phew_sdpa",
            ctypes.c_void_p(q._t.data_ptr()), ctypes.c_void_p(k._t.data_ptr()),
            ctypes.c_void_p(v._t.data_ptr()), ctypes.c_void_p(out._t.data_ptr()),
            B * H, L, D, ctypes.c_float(scale), 1 if causal else 0, q.dtype.code,
            ctypes.c_void_p(error_flag().data_ptr()), _stream(),
        )
        return out
    s = matmul(q, swapaxes(k, -1, -2)) * float(scale)
    if causal:
        s = s + causal_mask(q.shape[-2], k.shape[-2], s.dtype)
    elif mask is not None:
        mk = mask if isinstance(mask, array) else array(mask)
        s = s + (mk if mk.dtype is s.dtype else astype(mk, s.dtype))
    p = softmax(s, axis=-1)
    return matmul(p, v)
