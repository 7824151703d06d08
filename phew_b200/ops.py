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


def _param(p, x, cols: int, what: str):
    if p is None:
        return None, None
    a = asarray_device(p)
    if a.dtype is not x.dtype:
        a = a.astype(x.dtype)
    if a.shape != (cols,):
        raise ValueError(f"{what} shape {a.shape} != ({cols},)")
    return a, ctypes.c_void_p(a._t.data_ptr())


def layer_norm(x, weight=None, bias=None, eps: float = 1e-5) -> array:
    """``mx.fast.layer_norm(x, weight, bias, eps)`` over the last axis.

    n = cast((x - mean) * rsqrt(var + eps)) with fp32 mean and biased
    variance, y = cast(weight * n + bias); weight / bias None -> omitted.
    Node FastLayerNorm (phew ``ir/ops.py:165-168``), matched by
    ``rules/primitive_subst.py:246-333``, emitted at ``emit/codegen.py:406-411``.
    """
    x = asarray_device(x)
    if x.dtype.code is None:
        raise TypeError(f"layer_norm: unsupported dtype {x.dtype.name}")
    cols = x.shape[-1]
    rows = x.size // max(cols, 1)
    w, wptr = _param(weight, x, cols, "layer_norm: weight")
    b, bptr = _param(bias, x, cols, "layer_norm: bias")
    out = empty(x.shape, x.dtype)
    if x.size:
        _native.call(
            "phew_layer_norm", ctypes.c_void_p(x._t.data_ptr()), wptr, bptr,
            ctypes.c_void_p(out._t.data_ptr()), rows, cols, ctypes.c_float(eps), x.dtype.code,
            _stream(),
        )
    _ = (w, b)
    return out


def rope(x, dims: int, *, traditional: bool = False, base: float = 10000.0, scale: float = 1.0,
         offset: int = 0) -> array:
    """``mx.fast.rope(x, dims, traditional=, base=, scale=, offset=)``.

    Positions run along the second-to-last axis from `offset`; the first
    `dims` features of the last axis rotate in pairs (i, i + dims/2), or
    (2i, 2i+1) when `traditional`, by position * scale * base^(-2i/dims).
    Node FastRoPE (phew ``ir/ops.py:172-179``), matched by
    ``rules/primitive_subst.py:339-407``, emitted at ``emit/codegen.py:413-419``.
    """
    x = asarray_device(x)
    if x.dtype.code is None:
        raise TypeError(f"rope: unsupported dtype {x.dtype.name}")
    D = x.shape[-1] if x.ndim else 1
    L = x.shape[-2] if x.ndim >= 2 else 1
    rows = x.size // max(D, 1)
    out = empty(x.shape, x.dtype)
    if x.size:
        _native.call(
            "phew_rope", ctypes.c_void_p(x._t.data_ptr()), ctypes.c_void_p(out._t.data_ptr()),
            rows, D, L, int(dims), 1 if traditional else 0, ctypes.c_float(base),
            ctypes.c_float(scale), int(offset), x.dtype.code, _stream(),
        )
    return out


def dequantize(w, scales, biases, group_size: int = 64, bits: int = 4) -> array:
    """``mx.dequantize``: affine group-wise codes packed 32/bits per uint32
    along the last axis -> scales * q + biases in the scales' dtype."""
    import torch

    w = asarray_device(w)
    s = asarray_device(scales)
    b = asarray_device(biases)
    if s.dtype.code is None:
        raise TypeError(f"dequantize: unsupported scale dtype {s.dtype.name}")
    if b.dtype is not s.dtype:
        b = b.astype(s.dtype)
    per = 32 // int(bits)
    cols = w.shape[-1] * per
    rows = w.size // max(w.shape[-1], 1)
    if s.shape[-1] * int(group_size) != cols or s.size != rows * (cols // int(group_size)):
        raise ValueError(f"dequantize: scales {s.shape} do not match codes {w.shape} at "
                         f"group_size {group_size}, bits {bits}")
    wt = w._t if w._t.dtype in (torch.uint32, torch.int32) else w._t.to(torch.int32)
    out = empty(tuple(w.shape[:-1]) + (cols,), s.dtype)
    if out.size:
        _native.call(
            "phew_dequantize", ctypes.c_void_p(wt.data_ptr()), ctypes.c_void_p(s._t.data_ptr()),
            ctypes.c_void_p(b._t.data_ptr()), ctypes.c_void_p(out._t.data_ptr()), rows, cols,
            int(group_size), int(bits), s.dtype.code, _stream(),
        )
    return out


def quantized_matmul(x, w, scales=None, biases=None, transpose: bool = True, group_size: int = 64,
                     bits: int = 4, **_) -> array:
    """``mx.quantized_matmul(x, w, scales, biases, transpose=, group_size=, bits=)``:
    x @ dequantize(w).T (transpose) or x @ dequantize(w).  The weight is
    expanded by ``phew_dequantize`` and the product runs on the tcgen05
    GEMM.  Like MLX it needs the scales (the reference's QuantizationPass
    emits two-argument calls, ``rules/quantization.py:62-69``, which raise
    here as they would in MLX)."""
    from .mx.core import swapaxes

    if scales is None or biases is None:
        raise TypeError("quantized_matmul: scales and biases are required for affine quantization")
    wd = dequantize(w, scales, biases, group_size, bits)
    xd = asarray_device(x)
    if xd.dtype is not wd.dtype:
        xd = xd.astype(wd.dtype)
    return matmul(xd, swapaxes(wd, -1, -2) if transpose else wd)


def quantized_sdpa(q, k, v, scale_k, biases_k, scale_v, biases_v, *, scale: float = 1.0,
                   bits: int = 4, group_size: int = 64, mask=None) -> array:
    """``mx.fast.quantized_scaled_dot_product_attention``: k and v quantised
    along the head dimension, expanded by ``phew_dequantize``, then the
    attention kernel."""
    kd = dequantize(k, scale_k, biases_k, group_size, bits)
    vd = dequantize(v, scale_v, biases_v, group_size, bits)
    qd = asarray_device(q)
    if qd.dtype is not kd.dtype:
        qd = qd.astype(kd.dtype)
    return scaled_dot_product_attention(qd, kd, vd, scale=scale, mask=mask)


def quantize(w, group_size: int = 64, bits: int = 4):
    """``mx.quantize``: affine group-wise quantisation along the last axis ->
    (codes packed 32/bits per uint32, scales, biases), on ``phew_quantize``.
    Per group: scale = (max - min) / (2^bits - 1) (at least 1e-8, rounded to
    w's dtype), bias = min (rounded), q = round((w - bias) / scale) clipped
    to [0, 2^bits - 1]."""
    from . import dtypes as dt

    w = asarray_device(w)
    if w.dtype.code is None:
        raise TypeError(f"quantize: floating-point weights required, got {w.dtype.name}")
    g, nb = int(group_size), int(bits)
    per = 32 // nb
    cols = w.shape[-1]
    if cols % g or g % per:
        raise ValueError("quantize: the last axis must be a multiple of group_size, and "
                         "group_size of 32/bits")
    if not w._t.is_contiguous():
        from .mx.core import contiguous_copy

        w = contiguous_copy(w)
    rows = w.size // cols
    shp = tuple(w.shape[:-1])
    wq = empty(shp + (cols // per,), dt.uint32)
    sc = empty(shp + (cols // g,), w.dtype)
    bi = empty(shp + (cols // g,), w.dtype)
    _native.call("phew_quantize", ctypes.c_void_p(w._t.data_ptr()), ctypes.c_void_p(wq._t.data_ptr()),
                 ctypes.c_void_p(sc._t.data_ptr()), ctypes.c_void_p(bi._t.data_ptr()),
                 ctypes.c_int64(rows), ctypes.c_int64(cols), g, nb, w.dtype.code, _stream())
    return wq, sc, bi


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


def _two_axes(t) -> bool:
    """A 4-D operand whose two batch strides are both non-zero or both zero
    (batched over both axes or broadcast over both), as phew_gemm_batched2
    takes them."""
    return t.ndim == 4 and (t.stride(0) == 0) == (t.stride(1) == 0)


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

    ``row_scale=True`` returns ``(a @ b) * rsqrt(mean(a*a, -1) + eps)`` (the
    normed matmul of ``rules/primitive_subst.py:156-240``): one pass over
    ``a`` for the per-row factor, then the GEMM with the factor applied in its
    epilogue.
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
    tb = b._t.expand(*batch_shape, K, N)
    layout = None
    if (tb.stride(-1) == 1 or N == 1) and (K == 1 or tb.stride(-2) >= N):
        layout, ldb = 0, (tb.stride(-2) if K > 1 else N)
    elif (tb.stride(-2) == 1 or K == 1) and (N == 1 or tb.stride(-1) >= K):
        layout, ldb = 1, (tb.stride(-1) if N > 1 else K)
    if (not row_scale and len(batch_shape) == 2 and M > 1 and K > 1 and layout is not None
            and ta.stride(-1) == 1 and ta.stride(-2) >= K
            and (_collapse_batch(ta, batch_shape) is None or _collapse_batch(tb, batch_shape) is None)
            and _two_axes(ta) and _two_axes(tb)):
        # (batch, head) views that no single batch stride describes -- q, k
        # and v sliced out of a fused qkv projection: read in place
        out = empty(tuple(batch_shape) + (M, N), res)
        if out.size:
            _native.call(
                "phew_gemm_batched2",
                ctypes.c_void_p(ta.data_ptr()), ctypes.c_void_p(tb.data_ptr()),
                ctypes.c_void_p(out._t.data_ptr()),
                M, N, K, batch_shape[0], batch_shape[1], ta.stride(-2), ldb, N,
                ta.stride(0), ta.stride(1), tb.stride(0), tb.stride(1), M * N,
                layout, res.code, res.code,
                ctypes.c_void_p(error_flag().data_ptr()), _stream(),
            )
        if squeeze_a:
            out = reshape(out, out.shape[:-2] + (N,))
        if squeeze_b:
            out = reshape(out, out.shape[:-1])
        return out
    if ta.stride(-1) != 1 and K > 1 or _collapse_batch(ta, batch_shape) is None:
        ta = contiguous_copy(array._wrap(ta))._t
    lda = ta.stride(-2) if M > 1 else K
    sa = _collapse_batch(ta, batch_shape)

    if layout == 1 and _collapse_batch(tb, batch_shape) is None:
        # A K-major B (a transposed view, e.g. k.transpose(0, 1, 3, 2) of a
        # fused qkv projection) whose batch dims do not collapse to one
        # stride: copy it in its own (N, K) layout -- rows of K contiguous
        # elements, 16-byte vector copies -- and keep the K-major GEMM form,
        # instead of materialising the transpose element by element.
        tb = contiguous_copy(array._wrap(tb.transpose(-1, -2)))._t.transpose(-1, -2)
        ldb = K
    elif layout is None or _collapse_batch(tb, batch_shape) is None:
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
    from .mx.core import astype, contiguous_copy, softmax, swapaxes

    q = asarray_device(q, contiguous=False)
    k = asarray_device(k, contiguous=False)
    v = asarray_device(v, contiguous=False)
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
        # [B][H][L][D] views read in place when each has unit column stride
        # and 16-byte row / head / batch strides (q, k, v of a fused qkv
        # projection); anything else is copied first
        ts = []
        for x in (q, k, v):
            t = x._t
            st = (t.stride(2), t.stride(1), t.stride(0))
            if t.stride(3) != 1 or any(s_ <= 0 or s_ % 8 for s_ in st) or t.data_ptr() % 16:
                t = contiguous_copy(array._wrap(t))._t
                st = (D, L * D, H * L * D)
            ts.append((t, (ctypes.c_int64 * 3)(*st)))
        (tq, sq), (tk, sk), (tv, sv) = ts
        _native.call(
            "phew_sdpa_strided",
            ctypes.c_void_p(tq.data_ptr()), ctypes.c_void_p(tk.data_ptr()),
            ctypes.c_void_p(tv.data_ptr()), ctypes.c_void_p(out._t.data_ptr()),
            B, H, L, D, sq, sk, sv, ctypes.c_float(scale), 1 if causal else 0, q.dtype.code,
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
