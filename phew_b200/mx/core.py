"""Arrays and ops of the ``phew_b200.mx`` namespace.

This is the surface that phew's emitted ``output_source`` and a user's
harness function call: the subset of ``mlx.core`` that the candidate path
uses (phew ``emit/codegen.py:94-476``), executed eagerly on the current CUDA
device by this package's kernels:

* elementwise ops and casts -> one NVRTC kernel emitted by
  ``SubgraphCUDACodegen`` per (op, shapes, dtypes), Python scalars inlined as
  constants of the array's dtype (MLX weak scalars);
* reductions, softmax, rms_norm, strided copies -> the hand-written kernels
  of ``libphew_b200.so``;
* ``@`` / ``matmul`` and SDPA -> the tcgen05 kernels (``phew_b200.ops``).

PyTorch only allocates device memory (``torch.empty``) and provides the
current stream; no torch compute kernel runs on these paths.
"""

from __future__ import annotations

import builtins
import ctypes
import functools
import math
import numbers
import threading
import weakref
from typing import Any, Sequence

import numpy as np
import torch

from .. import _native
from .. import dtypes as dt
from ..dtypes import (  # noqa: F401  (re-exported as mx.float16 ...)
    Dtype,
    bfloat16,
    bool_,
    complex64,
    float16,
    float32,
    float64,
    int8,
    int16,
    int32,
    int64,
    uint8,
    uint16,
    uint32,
    uint64,
)
from ..emit.cuda_codegen import SubgraphCUDACodegen
from ..graph import NodeSpec
from ..kernel import CudaKernel

_DEVICE: torch.device | None = None


def device() -> torch.device:
    global _DEVICE
    if _DEVICE is None:
        if not torch.cuda.is_available():
            raise RuntimeError("phew_b200.mx needs a CUDA device (there is no CPU fallback)")
        idx = torch.cuda.current_device()
        _native.call("phew_init", idx)
        _DEVICE = torch.device("cuda", idx)
    return _DEVICE


def _stream() -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


@functools.lru_cache(maxsize=None)
def sm_count() -> int:
    info = _native.DeviceInfo()
    _native.call("phew_device_query", torch.cuda.current_device(), ctypes.byref(info))
    return int(info.sm_count)


def elementwise_threads(numel: int) -> int:
    """Total threads for an emitted grid-stride elementwise kernel.

    One thread per 8 elements (one 16-byte vector of a 16-bit type), capped
    at eight waves of 2048 threads on every SM; threads loop over the rest.
    (Measured on the fp16 (4096, 8192) chain: 1 wave 4852 GB/s, 2 waves 5110,
    4 waves 5278, 8 waves 5450.)
    """
    want = builtins.max(1, -(-numel // 8))
    cap = sm_count() * 2048 * 8
    return builtins.min(want, cap)


# ---------------------------------------------------------------------------
# array
# ---------------------------------------------------------------------------


class array:
    """A device array (storage: a CUDA torch tensor, possibly a strided view)."""

    __slots__ = ("_t", "__weakref__")

    def __init__(self, val: Any, dtype: Any = None) -> None:
        if isinstance(val, array):
            t = val._t if dtype is None else val.astype(dtype)._t
        elif isinstance(val, torch.Tensor):
            t = val if val.is_cuda else val.to(device())
            if dtype is not None and dt.from_any(dtype).torch != t.dtype:
                t = array(t).astype(dtype)._t
        else:
            t = _host_to_device(val, dtype)
        object.__setattr__(self, "_t", t)

    @classmethod
    def _wrap(cls, t: torch.Tensor) -> "array":
        a = object.__new__(cls)
        object.__setattr__(a, "_t", t)
        return a

    # -- metadata ------------------------------------------------------------
    @property
    def shape(self) -> tuple:
        return tuple(self._t.shape)

    @property
    def dtype(self) -> Dtype:
        return dt.from_any(self._t.dtype)

    @property
    def size(self) -> int:
        return self._t.numel()

    @property
    def ndim(self) -> int:
        return self._t.dim()

    @property
    def itemsize(self) -> int:
        return self._t.element_size()

    @property
    def nbytes(self) -> int:
        return self.size * self.itemsize

    def __len__(self) -> int:
        if self.ndim == 0:
            raise TypeError("len() of a 0-d array")
        return self.shape[0]

    def __repr__(self) -> str:
        return f"array(shape={self.shape}, dtype={self.dtype!r})"

    # -- host interop ----------------------------------------------------------
    def __array__(self, dtype=None, copy=None):
        out = to_numpy(self)
        return out.astype(dtype) if dtype is not None else out

    def item(self):
        return to_numpy(self).reshape(()).item()

    def tolist(self):
        return to_numpy(self).tolist()

    # -- views / layout ----------------------------------------------------------
    @property
    def T(self) -> "array":
        return transpose(self)

    def transpose(self, *axes) -> "array":
        if len(axes) == 1 and isinstance(axes[0], (list, tuple)):
            axes = tuple(axes[0])
        return transpose(self, axes or None)

    def swapaxes(self, a: int, b: int) -> "array":
        return swapaxes(self, a, b)

    def reshape(self, *shape) -> "array":
        if len(shape) == 1 and isinstance(shape[0], (list, tuple)):
            shape = tuple(shape[0])
        return reshape(self, shape)

    def flatten(self) -> "array":
        return reshape(self, (-1,))

    def astype(self, dtype) -> "array":
        return astype(self, dtype)

    def __getitem__(self, idx) -> "array":
        return array._wrap(self._t[idx])

    # -- reductions --------------------------------------------------------------
    def sum(self, axis=None, keepdims=False):
        return sum(self, axis=axis, keepdims=keepdims)

    def mean(self, axis=None, keepdims=False):
        return mean(self, axis=axis, keepdims=keepdims)

    def max(self, axis=None, keepdims=False):
        return max(self, axis=axis, keepdims=keepdims)

    def min(self, axis=None, keepdims=False):
        return min(self, axis=axis, keepdims=keepdims)

    # -- operators ---------------------------------------------------------------
    def __add__(self, o):
        return _binary("add", self, o)

    def __radd__(self, o):
        return _binary("add", o, self)

    def __sub__(self, o):
        return _binary("sub", self, o)

    def __rsub__(self, o):
        return _binary("sub", o, self)

    def __mul__(self, o):
        return _binary("mul", self, o)

    def __rmul__(self, o):
        return _binary("mul", o, self)

    def __truediv__(self, o):
        return _binary("div", self, o)

    def __rtruediv__(self, o):
        return _binary("div", o, self)

    def __floordiv__(self, o):
        return _binary("floor_divide", self, o)

    def __mod__(self, o):
        return _binary("remainder", self, o)

    def __pow__(self, o):
        return _binary("power", self, o)

    def __rpow__(self, o):
        return _binary("power", o, self)

    def __neg__(self):
        return _unary("negative", self)

    def __abs__(self):
        return _unary("abs", self)

    def __eq__(self, o):  # noqa: D105  (elementwise, as in MLX)
        return _binary("eq", self, o, out_bool=True)

    def __ne__(self, o):
        return _binary("ne", self, o, out_bool=True)

    def __lt__(self, o):
        return _binary("lt", self, o, out_bool=True)

    def __le__(self, o):
        return _binary("le", self, o, out_bool=True)

    def __gt__(self, o):
        return _binary("gt", self, o, out_bool=True)

    def __ge__(self, o):
        return _binary("ge", self, o, out_bool=True)

    __hash__ = object.__hash__

    def __matmul__(self, o):
        return matmul(self, o)

    def __rmatmul__(self, o):
        return matmul(o, self)


# ---------------------------------------------------------------------------
# host <-> device
# ---------------------------------------------------------------------------

_scalar_cache: dict[tuple, torch.Tensor] = {}


def _host_to_device(val: Any, dtype: Any) -> torch.Tensor:
    d = dt.from_any(dtype) if dtype is not None else None
    if isinstance(val, (bool, numbers.Number)) and not isinstance(val, np.ndarray):
        if d is None:
            d = bool_ if isinstance(val, bool) else (int32 if isinstance(val, int) else float32)
        key = (type(val).__name__, val if not (isinstance(val, float) and math.isnan(val)) else "nan", d.name)
        t = _scalar_cache.get(key)
        if t is None:
            t = _from_numpy(np.asarray(val).astype(np.float64 if d.kind == "f" else None), d)
            _scalar_cache[key] = t
        return t
    a = np.asarray(val)
    if d is None:
        if a.dtype == np.float64:
            d = float32
        elif a.dtype == np.int64 and not isinstance(val, np.ndarray):
            d = int32
        else:
            d = dt.from_any(a.dtype)
    return _from_numpy(a, d)


def _from_numpy(a: np.ndarray, d: Dtype) -> torch.Tensor:
    a = np.asarray(a)
    if d.kind == "f" and a.dtype != d.np:
        # float64 and other floats round through fp32, as inlined literals do
        a = a.astype(np.float32) if a.dtype.kind == "f" or a.dtype == bfloat16.np else a
    host = np.ascontiguousarray(a.astype(d.np))
    if d is bfloat16:
        t = torch.from_numpy(host.view(np.int16)).view(torch.bfloat16)
    else:
        t = torch.from_numpy(host)
    return t.to(device(), non_blocking=False)


def to_numpy(a: "array") -> np.ndarray:
    t = a._t.detach()
    if t.dtype == torch.bfloat16:
        host = t.contiguous().cpu().view(torch.int16).numpy().view(bfloat16.np)
        return host
    return t.cpu().numpy()


def asarray_device(x: Any, contiguous: bool = True) -> array:
    """Coerce to an `array` on the device, materialising strided views."""
    a = x if isinstance(x, array) else array(x)
    if contiguous and not a._t.is_contiguous():
        a = contiguous_copy(a)
    return a


def empty(shape: Sequence[int], dtype: Any) -> array:
    d = dt.from_any(dtype)
    return array._wrap(torch.empty(tuple(shape), dtype=d.torch, device=device()))


def contiguous_copy(a: array) -> array:
    """Materialise a strided view with the strided-copy kernel."""
    t = a._t
    out = torch.empty(t.shape, dtype=t.dtype, device=t.device)
    if t.numel() == 0:
        return array._wrap(out)
    # Drop size-1 dims and merge nothing: the kernel takes up to 8 dims.
    shape = [s for s in t.shape]
    strides = list(t.stride())
    if len(shape) == 0:
        shape, strides = [1], [1]
    if len(shape) > 8:
        keep = [(s, st) for s, st in zip(shape, strides) if s != 1]
        shape = [s for s, _ in keep] or [1]
        strides = [st for _, st in keep] or [1]
        if len(shape) > 8:
            raise NotImplementedError("strided copy of more than 8 non-unit dims")
    n = len(shape)
    cs = (ctypes.c_int64 * n)(*shape)
    cst = (ctypes.c_int64 * n)(*strides)
    _native.call(
        "phew_copy_strided",
        ctypes.c_void_p(t.data_ptr()),
        ctypes.c_void_p(out.data_ptr()),
        n, cs, cst, t.element_size(), _stream(),
    )
    return array._wrap(out)


# ---------------------------------------------------------------------------
# elementwise ops through the fused-chain emitter
# ---------------------------------------------------------------------------

_kernel_cache: dict[tuple, tuple] = {}


def _broadcast_shapes(*shapes) -> tuple:
    nd = builtins_max((len(s) for s in shapes), default=0)
    out = []
    for i in range(nd):
        d = 1
        for s in shapes:
            p = (1,) * (nd - len(s)) + tuple(s)
            if p[i] != 1:
                if d != 1 and d != p[i]:
                    raise ValueError(f"shapes {shapes} cannot be broadcast")
                d = p[i]
        out.append(d)
    return tuple(out)


builtins_max = max  # shadowed below by mx.max
builtins_min = min
builtins_sum = sum


def _elementwise(op: str, operands: list, out_dtype: Dtype | None = None,
                 out_bool: bool = False) -> array:
    """Run `op` over operands (arrays or Python scalars) with one emitted kernel."""
    arrays = [x for x in operands if isinstance(x, array)]
    if not arrays:
        raise TypeError(f"{op}: needs at least one array operand")
    # Result dtype: arrays promote; Python scalars are weak.
    res = arrays[0].dtype
    for a in arrays[1:]:
        res = dt.promote(res, a.dtype)
    for x in operands:
        if not isinstance(x, array):
            res = dt.scalar_dtype(x, res)
    compute_dt = res
    node_dt = bool_ if out_bool else (out_dtype or res)
    shape = _broadcast_shapes(*[a.shape for a in arrays])
    if _tracing() and _numel(shape) > 0:
        return _Lazy._new(op, operands, compute_dt, node_dt, shape)
    key_parts = []
    for x in operands:
        if isinstance(x, array):
            key_parts.append(("a", x.shape, x.dtype.name))
        else:
            key_parts.append(("s", type(x).__name__, repr(x)))
    key = (op, tuple(key_parts), compute_dt.name, node_dt.name)
    entry = _kernel_cache.get(key)
    if entry is None:
        entry = _build_elementwise(op, operands, compute_dt, node_dt, shape)
        _kernel_cache[key] = entry
    kern, in_positions = entry
    ins = [asarray_device(operands[i]) for i in in_positions]
    out = kern(
        inputs=ins,
        output_shapes=[shape],
        output_dtypes=[node_dt],
        grid=(elementwise_threads(_numel(shape)), 1, 1),
        threadgroup=(256, 1, 1),
    )
    return out[0]


# ---------------------------------------------------------------------------
# deferred elementwise results inside mx.compile
# ---------------------------------------------------------------------------
#
# Inside a function wrapped by ``mx.compile`` elementwise ops do not launch:
# they return `_Lazy` arrays, nodes of a pending DAG.  The first read of a
# node's storage (any non-elementwise op, a view, a host copy, the function's
# return) emits the node and every pending elementwise node it depends on as
# ONE fused kernel (the same per-element code as the fusion pass's chains:
# every node rounded to its own dtype, so the values are those of op-by-op
# evaluation) and keeps the result.  A pending node read by two different
# materialisations is computed in both (elementwise recompute is cheaper
# than a round trip through HBM).

_trace = threading.local()


def _tracing() -> bool:
    return getattr(_trace, "depth", 0) > 0


class _Lazy(array):
    """A pending elementwise result (see the section comment)."""

    __slots__ = ("_op", "_shape", "_dtype", "_mt")

    @classmethod
    def _new(cls, op, operands, compute_dt, node_dt, shape) -> "_Lazy":
        a = object.__new__(cls)
        object.__setattr__(a, "_op", (op, tuple(operands), compute_dt, node_dt))
        object.__setattr__(a, "_shape", tuple(int(x) for x in shape))
        object.__setattr__(a, "_dtype", node_dt)
        object.__setattr__(a, "_mt", None)
        return a

    @property
    def _t(self) -> torch.Tensor:  # type: ignore[override]
        if self._mt is None:
            _materialize(self)
        return self._mt

    @property
    def pending(self) -> bool:
        return self._mt is None

    @property
    def _pending_dag(self) -> bool:
        """Pending, and an elementwise node (not a deferred row reduction)."""
        return self._mt is None and self._op[0] != _ROW_REDUCE

    @property
    def shape(self) -> tuple:
        return self._shape

    @property
    def dtype(self) -> Dtype:
        return self._dtype

    @property
    def size(self) -> int:
        return _numel(self._shape)

    @property
    def ndim(self) -> int:
        return len(self._shape)

    @property
    def itemsize(self) -> int:
        return self._dtype.size


# A last-axis keepdims reduction of a pending DAG is deferred as well (its
# `_op` is (_ROW_REDUCE, opname, source)): when the DAG that reads it covers
# the same rows (the tail of an RMS or layer norm), reduction and tail run as
# one row kernel (`_fused_row_map`); any other read computes it alone.
_ROW_REDUCE = "__row_reduce__"


def _row_reduce_plan(red: int) -> tuple[int, int]:
    """(threads per row, rows per block) of ``reduce_rows_kernel`` in
    csrc/rows.cu for rows of `red` elements: the fused forms use the same
    mapping, so their sums are added in the same order."""
    tpr = 256 if red >= 1024 else 32
    return tpr, (4 if tpr == 32 else 1)


def _fused_dag(root: "_Lazy"):
    """NodeSpecs of the pending DAG under `root` (topological order), its
    external inputs (specs and arrays, in first-visit order) and a key that
    identifies the DAG's structure for the kernel cache."""
    chain: list = []
    ext_specs: list = []
    ext_arrays: list = []
    key: list = []
    memo: dict[int, tuple] = {}

    def visit(x):
        hit = memo.get(id(x))
        if hit is not None:
            return hit
        if isinstance(x, _Lazy) and x._pending_dag:
            op, operands, cdt, ndt = x._op
            args, arg_keys = [], []
            for o in operands:
                if isinstance(o, array):
                    spec, k = visit(o)
                    if o.dtype is not cdt and op != "where":
                        spec = NodeSpec("Cast", o.shape, cdt.name, inputs=[spec.id], target_dtype=cdt.name)
                        chain.append(spec)
                        key.append(("cast", k, cdt.name))
                        k = len(key) - 1
                else:
                    spec = NodeSpec("Constant", (), cdt.name, value=o)
                    chain.append(spec)
                    key.append(("const", cdt.name, type(o).__name__, repr(o)))
                    k = len(key) - 1
                args.append(spec)
                arg_keys.append(k)
            node = NodeSpec("Elementwise", x._shape, ndt.name, inputs=[a.id for a in args], op=op)
            chain.append(node)
            key.append(("ew", op, x._shape, ndt.name, tuple(arg_keys)))
        else:
            node = NodeSpec("Input", x.shape, x.dtype.name)
            ext_specs.append(node)
            ext_arrays.append(x)
            key.append(("in", x.shape, x.dtype.name))
        memo[id(x)] = (node, len(key) - 1)
        return memo[id(x)]

    try:
        root_spec, _ = visit(root)
    finally:
        # `visit` refers to itself through its closure cell; break that cycle
        # so the arrays it reaches are freed by reference counting, not left
        # for the cyclic collector (they can be tens of GB).
        visit = None  # noqa: F841
    return chain, ext_specs, ext_arrays, root_spec, tuple(key)


def _materialize(root: "_Lazy") -> None:
    if root._op[0] == _ROW_REDUCE:
        _, opname, src = root._op
        out = _fused_reduce(opname, src, True) if isinstance(src, _Lazy) and src._pending_dag else None
        if out is None:
            out = _reduce_now(opname, array._wrap(asarray_device(src)._t), -1, True)
        object.__setattr__(root, "_mt", out._t)
        object.__setattr__(root, "_op", None)
        return
    chain, ext_specs, ext_arrays, root_spec, key = _fused_dag(root)
    # Deferred row reductions read by this DAG: the last one whose rows are
    # the DAG's own runs inside its kernel; the others are computed first.
    rows = [i for i, x in enumerate(ext_arrays) if isinstance(x, _Lazy) and x.pending]
    for i in reversed(rows):
        if _fused_row_map(root, chain, ext_specs, ext_arrays, root_spec, key, i):
            return
    ckey = ("fused", key)
    kern = _kernel_cache.get(ckey)
    if kern is None:
        src, in_names, out_names = SubgraphCUDACodegen().emit(chain, ext_specs, [root_spec])
        kern = CudaKernel(f"phew_fused_{len(chain)}", in_names, out_names, src)
        _kernel_cache[ckey] = kern
    out = kern(
        inputs=[asarray_device(a) for a in ext_arrays],
        output_shapes=[root._shape],
        output_dtypes=[root._dtype],
        grid=(elementwise_threads(_numel(root._shape)), 1, 1),
        threadgroup=(256, 1, 1),
    )
    object.__setattr__(root, "_mt", out[0]._t)
    object.__setattr__(root, "_op", None)


def _row_map_parts(root, chain, ext_specs, ext_arrays, root_spec, key, i):
    """(cache key, ``emit_row_map`` arguments, kernel input arrays) for
    `root`, whose DAG reads the deferred row reduction ``ext_arrays[i]``; None
    when the reduction's source does not cover the same rows."""
    m = ext_arrays[i]
    _, opname, src = m._op
    if root.ndim < 1 or tuple(src.shape) != tuple(root.shape) or root.size == 0:
        return None
    if isinstance(src, _Lazy) and src.pending and not src._pending_dag:
        return None  # a reduction of a deferred reduction: computed on its own
    tpr, rpb = _row_reduce_plan(root.shape[-1])
    rchain, rext_specs, rext_arrays, rroot_spec, rkey = _fused_dag(src)
    # One kernel only pays when the chain re-reads a full-size input of the
    # reduction (x in an RMS or layer norm): then that input crosses HBM once
    # instead of twice.  With disjoint inputs the separate reduce and chain
    # kernels move the same bytes, faster.
    full = tuple(root.shape)
    shared = {id(x) for x in rext_arrays if tuple(x.shape) == full} & {
        id(x) for k, x in enumerate(ext_arrays) if k != i and tuple(x.shape) == full}
    if not shared:
        return None
    slots: dict = {}
    arrays: list = []
    where: dict = {}
    pairs = list(zip(rext_specs, rext_arrays)) + [
        (sp, x) for k, (sp, x) in enumerate(zip(ext_specs, ext_arrays)) if k != i]
    for sp, x in pairs:
        j = where.get(id(x))
        if j is None:
            j = where[id(x)] = len(arrays)
            arrays.append(x)
        slots[sp.id] = j
    layout = (tuple(slots[sp.id] for sp in rext_specs),
              tuple(slots.get(sp.id, -1) for sp in ext_specs))
    ckey = ("row_map", opname, rkey, key, i, layout, tpr, rpb)
    args = (rchain, rext_specs, rroot_spec, opname, chain, ext_specs, root_spec, ext_specs[i],
            slots, tpr, rpb)
    return ckey, args, arrays


def _fused_row_map(root, chain, ext_specs, ext_arrays, root_spec, key, i) -> bool:
    """Materialise `root`, whose DAG reads the deferred row reduction
    ``ext_arrays[i]``, as one row kernel (``emit_row_map``): the reduction
    and the chain that reads it over the same rows; False when it cannot."""
    parts = _row_map_parts(root, chain, ext_specs, ext_arrays, root_spec, key, i)
    if parts is None:
        return False
    ckey, args, arrays = parts
    kern = _kernel_cache.get(ckey)
    if kern is None:
        try:
            src_code, in_names, out_names = SubgraphCUDACodegen().emit_row_map(*args)
        except ValueError:
            _kernel_cache[ckey] = False
            return False
        kern = CudaKernel(f"phew_row_{args[3]}_map_{len(args[0])}_{len(chain)}", in_names,
                          out_names, src_code)
        _kernel_cache[ckey] = kern
    if kern is False:
        return False
    tpr, rpb = args[-2], args[-1]
    # persistent row groups: enough blocks to fill the SMs, each walking
    # groups of rpb rows with a grid stride
    blocks = builtins_min(-(-(root.size // root.shape[-1]) // rpb), sm_count() * 8)
    out = kern(inputs=[asarray_device(x) for x in arrays], output_shapes=[root._shape],
               output_dtypes=[root._dtype], grid=(blocks * tpr, rpb, 1), threadgroup=(tpr, rpb, 1))
    object.__setattr__(root, "_mt", out[0]._t)
    object.__setattr__(root, "_op", None)
    return True


def _softmax_row_plan(cols: int, itemsize: int):
    """(threads per row, rows per block, vectors per thread) of the vector
    softmax kernel in csrc/rows.cu for rows of `cols` elements, or None when
    that kernel would take its loop form."""
    E = 16 // itemsize
    if cols % E:
        return None
    nvec = cols // E
    if nvec > 512 * 8:
        return None
    tpr = (((nvec + 3) // 4 + 31) // 32) * 32
    tpr = builtins_min(builtins_max(tpr, 32), 512)
    vpt = -(-nvec // tpr)
    rpb = 1 if tpr >= 128 else 128 // tpr
    return tpr, rpb, vpt


def _fused_softmax(a: "_Lazy"):
    """softmax over the last axis of a pending elementwise DAG, in one kernel
    that computes the DAG per row in registers; None when it cannot (the
    caller then materialises `a` and runs the plain softmax)."""
    plan = _softmax_row_plan(a.shape[-1], a.dtype.size)
    if plan is None or a.dtype.code is None:
        return None
    tpr, rpb, vpt = plan
    chain, ext_specs, ext_arrays, root_spec, key = _fused_dag(a)
    ins = [asarray_device(x) for x in ext_arrays]
    if builtins.any(x._t.data_ptr() % 16 for x in ins):
        return None
    ckey = ("fused_softmax", key, plan)
    kern = _kernel_cache.get(ckey)
    if kern is None:
        try:
            src, in_names, out_names = SubgraphCUDACodegen().emit_softmax(
                chain, ext_specs, root_spec, tpr, rpb, vpt)
        except ValueError:
            _kernel_cache[ckey] = False
            return None
        kern = CudaKernel(f"phew_fused_softmax_{len(chain)}", in_names, out_names, src)
        _kernel_cache[ckey] = kern
    if kern is False:
        return None
    rows = a.size // a.shape[-1]
    blocks = -(-rows // rpb)
    return kern(inputs=ins, output_shapes=[a.shape], output_dtypes=[a.dtype],
                grid=(blocks * tpr, rpb, 1), threadgroup=(tpr, rpb, 1))[0]


def trace_enter() -> None:
    _trace.depth = getattr(_trace, "depth", 0) + 1


def trace_exit() -> None:
    _trace.depth = getattr(_trace, "depth", 1) - 1


def settle(x):
    """Materialise every pending array in `x` (an array or nested list /
    tuple / dict of them) and return the same structure of plain arrays."""
    if isinstance(x, _Lazy):
        return array._wrap(x._t)
    if isinstance(x, (list, tuple)):
        vals = [settle(v) for v in x]
        return type(x)(vals) if isinstance(x, list) else tuple(vals)
    if isinstance(x, dict):
        return {k: settle(v) for k, v in x.items()}
    return x


def _numel(shape) -> int:
    n = 1
    for s in shape:
        n *= int(s)
    return n


def _build_elementwise(op, operands, compute_dt: Dtype, node_dt: Dtype, shape):
    ext, chain, args, positions = [], [], [], []
    for i, x in enumerate(operands):
        if isinstance(x, array):
            n = NodeSpec("Input", x.shape, x.dtype.name)
            ext.append(n)
            positions.append(i)
            if x.dtype is not compute_dt and op not in ("where",):
                c = NodeSpec("Cast", x.shape, compute_dt.name, inputs=[n.id],
                             target_dtype=compute_dt.name)
                chain.append(c)
                n = c
            args.append(n)
        else:
            c = NodeSpec("Constant", (), compute_dt.name, value=x)
            chain.append(c)
            args.append(c)
    node = NodeSpec("Elementwise", shape, node_dt.name, inputs=[a.id for a in args], op=op)
    chain.append(node)
    src, in_names, out_names = SubgraphCUDACodegen().emit(chain, ext, [node])
    kern = CudaKernel(f"phew_ew_{op}", in_names, out_names, src)
    return kern, positions


def _binary(op: str, a, b, out_bool: bool = False) -> array:
    return _elementwise(op, [a, b], out_bool=out_bool)


def _unary(op: str, a) -> array:
    return _elementwise(op, [asarray_device(a, contiguous=False)])


def _make_unary(op):
    def f(x, *_, **__):
        return _unary(op, x)

    f.__name__ = op
    return f


for _op in (
    "exp", "log", "sqrt", "rsqrt", "sigmoid", "tanh", "abs", "negative", "square", "sin",
    "cos", "tan", "erf", "erfinv", "expm1", "log1p", "log2", "log10", "ceil", "floor",
    "round", "sign", "reciprocal", "arcsin", "arccos", "arctan", "arcsinh", "arccosh",
    "arctanh", "sinh", "cosh", "degrees", "radians", "logical_not",
):
    globals()[_op] = _make_unary(_op)


def _make_binary(op, out_bool=False):
    def f(a, b, *_, **__):
        return _binary(op, a, b, out_bool=out_bool)

    f.__name__ = op
    return f


add = _make_binary("add")
subtract = _make_binary("sub")
multiply = _make_binary("mul")
divide = _make_binary("div")
maximum = _make_binary("maximum")
minimum = _make_binary("minimum")
power = _make_binary("power")
logaddexp = _make_binary("logaddexp")
floor_divide = _make_binary("floor_divide")
remainder = _make_binary("remainder")
arctan2 = _make_binary("arctan2")
equal = _make_binary("eq", True)
not_equal = _make_binary("ne", True)
greater = _make_binary("gt", True)
greater_equal = _make_binary("ge", True)
less = _make_binary("lt", True)
less_equal = _make_binary("le", True)
logical_and = _make_binary("logical_and", True)
logical_or = _make_binary("logical_or", True)


def where(cond, a, b) -> array:
    c = cond if isinstance(cond, array) else array(cond)
    vals = [x for x in (a, b) if isinstance(x, array)]
    res = vals[0].dtype if vals else float32
    for v in vals[1:]:
        res = dt.promote(res, v.dtype)
    a2 = a if not isinstance(a, array) or a.dtype is res else astype(a, res)
    b2 = b if not isinstance(b, array) or b.dtype is res else astype(b, res)
    return _elementwise("where", [c, a2, b2], out_dtype=res)


def astype(a, dtype) -> array:
    d = dt.from_any(dtype)
    a = a if isinstance(a, array) else array(a)
    if a.dtype is d:
        return a
    key = ("cast", a.shape, a.dtype.name, d.name)
    entry = _kernel_cache.get(key)
    if entry is None:
        x = NodeSpec("Input", a.shape, a.dtype.name)
        c = NodeSpec("Cast", a.shape, d.name, inputs=[x.id], target_dtype=d.name)
        src, i, o = SubgraphCUDACodegen().emit([c], [x], [c])
        entry = (CudaKernel("phew_cast", i, o, src), [0])
        _kernel_cache[key] = entry
    kern, _ = entry
    return kern(inputs=[asarray_device(a)], output_shapes=[a.shape], output_dtypes=[d],
                grid=(elementwise_threads(a.size), 1, 1), threadgroup=(256, 1, 1))[0]


def silu(x):
    return _unary("silu", x)


def gelu(x):
    return _unary("gelu", x)


def relu(x):
    return _unary("relu", x)


# ---------------------------------------------------------------------------
# layout
# ---------------------------------------------------------------------------


def transpose(a, axes=None) -> array:
    a = a if isinstance(a, array) else array(a)
    if axes is None:
        axes = tuple(range(a.ndim - 1, -1, -1))
    axes = tuple(int(x) % builtins_max(a.ndim, 1) for x in axes)
    return array._wrap(a._t.permute(*axes))


def swapaxes(a, x: int, y: int) -> array:
    axes = list(range(a.ndim))
    x, y = x % a.ndim, y % a.ndim
    axes[x], axes[y] = axes[y], axes[x]
    return transpose(a, axes)


def reshape(a, shape) -> array:
    a = a if isinstance(a, array) else array(a)
    shape = tuple(int(s) for s in (shape if isinstance(shape, (list, tuple)) else (shape,)))
    src = a if a._t.is_contiguous() else contiguous_copy(a)
    return array._wrap(src._t.view(shape))


def expand_dims(a, axis) -> array:
    axes = axis if isinstance(axis, (list, tuple)) else [axis]
    t = a._t
    for ax in sorted(int(x) % (t.dim() + len(axes)) for x in axes):
        t = t.unsqueeze(ax)
    return array._wrap(t)


def squeeze(a, axis=None) -> array:
    t = a._t
    if axis is None:
        return array._wrap(t.squeeze())
    axes = axis if isinstance(axis, (list, tuple)) else [axis]
    for ax in sorted((int(x) % t.dim() for x in axes), reverse=True):
        t = t.squeeze(ax)
    return array._wrap(t)


def broadcast_to(a, shape) -> array:
    return array._wrap(a._t.expand(*shape))


# ---------------------------------------------------------------------------
# reductions
# ---------------------------------------------------------------------------


def _norm_axes(a: array, axis) -> tuple:
    if axis is None:
        return tuple(range(a.ndim))
    if isinstance(axis, (list, tuple)):
        return tuple(sorted(int(x) % a.ndim for x in axis))
    return (int(axis) % a.ndim,)


def _fused_reduce(opname: str, a: "_Lazy", keepdims: bool):
    """`opname` over the last axis of a pending elementwise DAG, in one kernel
    that computes each element as the reduction reads it; None when it
    cannot (the caller then materialises `a`)."""
    red = a.shape[-1]
    if red == 0 or a.size == 0:
        return None
    tpr, rpb = _row_reduce_plan(red)
    chain, ext_specs, ext_arrays, root_spec, key = _fused_dag(a)
    ckey = ("fused_reduce", opname, key)
    kern = _kernel_cache.get(ckey)
    if kern is None:
        try:
            src, in_names, out_names = SubgraphCUDACodegen().emit_reduce_rows(
                chain, ext_specs, root_spec, opname, keepdims, tpr, rpb)
        except ValueError:
            _kernel_cache[ckey] = False
            return None
        kern = CudaKernel(f"phew_fused_{opname}_{len(chain)}", in_names, out_names, src)
        _kernel_cache[ckey] = kern
    if kern is False:
        return None
    rows = a.size // red
    out_shape = tuple(a.shape[:-1]) + ((1,) if keepdims else ())
    blocks = -(-rows // rpb)
    return kern(inputs=[asarray_device(x) for x in ext_arrays], output_shapes=[out_shape],
                output_dtypes=[a.dtype], grid=(blocks * tpr, rpb, 1), threadgroup=(tpr, rpb, 1))[0]


def _reduce(opname: str, a, axis=None, keepdims=False) -> array:
    a = a if isinstance(a, array) else array(a)
    if a.dtype.code is None:
        raise NotImplementedError(f"{opname} over {a.dtype.name} arrays")
    last_axis = a.ndim >= 1 and _norm_axes(a, axis) == (a.ndim - 1,)
    if (_tracing() and last_axis and keepdims and a.size > 0
            and a.dtype in (float32, float16, bfloat16)
            and not (isinstance(a, _Lazy) and a.pending and not a._pending_dag)):
        m = object.__new__(_Lazy)
        object.__setattr__(m, "_op", (_ROW_REDUCE, opname, a))
        object.__setattr__(m, "_shape", tuple(a.shape[:-1]) + (1,))
        object.__setattr__(m, "_dtype", a.dtype)
        object.__setattr__(m, "_mt", None)
        return m
    return _reduce_now(opname, a, axis, keepdims)


def _reduce_now(opname: str, a: array, axis, keepdims: bool) -> array:
    """`opname` of `a` computed now (never deferred)."""
    if (isinstance(a, _Lazy) and a._pending_dag and a.ndim >= 1
            and _norm_axes(a, axis) == (a.ndim - 1,)):
        fused = _fused_reduce(opname, a, keepdims)
        if fused is not None:
            return fused
    axes = _norm_axes(a, axis)
    shape = a.shape
    out_shape_keep = tuple(1 if i in axes else s for i, s in enumerate(shape))
    out_shape = out_shape_keep if keepdims else tuple(s for i, s in enumerate(shape) if i not in axes)
    if not axes:
        return a
    contiguous_block = axes == tuple(range(axes[0], axes[-1] + 1))
    src = asarray_device(a)
    if not contiguous_block:
        rest = [i for i in range(a.ndim) if i not in axes]
        src = contiguous_copy(transpose(src, rest + list(axes)))
        shape = tuple(a.shape[i] for i in rest) + tuple(a.shape[i] for i in axes)
        lo = len(rest)
        axes = tuple(range(lo, a.ndim))
    outer = _numel(shape[: axes[0]])
    red = _numel(shape[axes[0] : axes[-1] + 1])
    inner = _numel(shape[axes[-1] + 1 :])
    out = empty(out_shape, a.dtype)
    if out.size == 0:
        return out
    if red == 0:
        fill = {"sum": 0.0, "mean": float("nan"), "prod": 1.0, "max": -math.inf, "min": math.inf}
        out._t.fill_(fill[opname])
        return out
    _native.call(
        "phew_reduce", _native.REDUCE_OPS[opname], ctypes.c_void_p(src._t.data_ptr()),
        ctypes.c_void_p(out._t.data_ptr()), outer, red, inner, a.dtype.code, _stream(),
    )
    return out


def sum(a, axis=None, keepdims=False, **_) -> array:  # noqa: A001
    return _reduce("sum", a, axis, keepdims)


def mean(a, axis=None, keepdims=False, **_) -> array:
    return _reduce("mean", a, axis, keepdims)


def max(a, axis=None, keepdims=False, **_) -> array:  # noqa: A001
    return _reduce("max", a, axis, keepdims)


def min(a, axis=None, keepdims=False, **_) -> array:  # noqa: A001
    return _reduce("min", a, axis, keepdims)


def prod(a, axis=None, keepdims=False, **_) -> array:
    return _reduce("prod", a, axis, keepdims)


def softmax(a, axis=-1, precise=False, **_) -> array:
    a = a if isinstance(a, array) else array(a)
    if a.dtype.code is None:
        raise NotImplementedError(f"softmax over {a.dtype.name} arrays")
    if isinstance(axis, (list, tuple)):
        if len(axis) != 1:
            raise NotImplementedError("softmax over several axes")
        axis = axis[0]
    ax = int(axis) % a.ndim
    if ax != a.ndim - 1:
        moved = swapaxes(a, ax, a.ndim - 1)
        return swapaxes(softmax(moved, axis=-1), ax, a.ndim - 1)
    if isinstance(a, _Lazy) and a._pending_dag:
        fused = _fused_softmax(a)
        if fused is not None:
            return fused
    src = asarray_device(a)
    out = empty(a.shape, a.dtype)
    cols = a.shape[-1] if a.ndim else 1
    rows = a.size // builtins_max(cols, 1)
    if a.size:
        _native.call(
            "phew_softmax", ctypes.c_void_p(src._t.data_ptr()), ctypes.c_void_p(out._t.data_ptr()),
            rows, cols, a.dtype.code, _stream(),
        )
    return out


# ---------------------------------------------------------------------------
# constructors, evaluation and compile
# ---------------------------------------------------------------------------


def zeros(shape, dtype=float32) -> array:
    d = dt.from_any(dtype)
    shape = (shape,) if isinstance(shape, int) else tuple(shape)
    return array._wrap(torch.zeros(shape, dtype=d.torch, device=device()))


def ones(shape, dtype=float32) -> array:
    d = dt.from_any(dtype)
    shape = (shape,) if isinstance(shape, int) else tuple(shape)
    return array._wrap(torch.ones(shape, dtype=d.torch, device=device()))


def full(shape, value, dtype=None) -> array:
    d = dt.from_any(dtype) if dtype is not None else (float32 if isinstance(value, float) else int32)
    shape = (shape,) if isinstance(shape, int) else tuple(shape)
    return array._wrap(torch.full(shape, value, dtype=d.torch, device=device()))


def zeros_like(a) -> array:
    return array._wrap(torch.zeros(a.shape, dtype=a._t.dtype, device=device()))


def ones_like(a) -> array:
    return array._wrap(torch.ones(a.shape, dtype=a._t.dtype, device=device()))


def eval(*args) -> None:  # noqa: A001  (MLX name)
    """Computes pending (deferred, inside ``mx.compile``) arrays among `args`
    (arrays or nested lists / tuples / dicts of them); others already are."""
    stack = list(args)
    while stack:
        x = stack.pop()
        if isinstance(x, _Lazy):
            x._t  # noqa: B018  (materialises)
        elif isinstance(x, (list, tuple)):
            stack.extend(x)
        elif isinstance(x, dict):
            stack.extend(x.values())


def async_eval(*args) -> None:
    eval(*args)


def synchronize(stream=None) -> None:
    torch.cuda.current_stream().synchronize()


def matmul(a, b) -> array:
    from ..ops import matmul as _mm

    return _mm(a, b)


def compile(fn=None, *, shapeless: bool = False, **_):  # noqa: A001  (MLX name)
    """``@mx.compile``: see :mod:`phew_b200.graphs` for the CUDA-graph capture."""
    from ..graphs import compile_function

    if fn is None:
        return lambda f: compile_function(f)
    return compile_function(fn)


class _Metal:
    @staticmethod
    def is_available() -> bool:
        return False


metal = _Metal()


def is_available() -> bool:
    return torch.cuda.is_available()


def device_info() -> dict:
    info = _native.DeviceInfo()
    _native.call("phew_device_query", torch.cuda.current_device(), ctypes.byref(info))
    return {
        "device_name": info.name.decode(),
        "architecture": f"sm_{info.cc_major}{info.cc_minor}",
        "sm_count": info.sm_count,
        "memory_size": info.hbm_bytes,
        "l2_cache_size": info.l2_bytes,
    }


_live_arrays = weakref.WeakSet()
