"""CUDA C++ source generator for fused elementwise subgraphs (NVRTC, sm_100a).

Stands in for ``SubgraphMSLCodegen`` (phew ``emit/msl_codegen.py:125-330``)
with the same call shape::

    source, input_names, output_names = SubgraphCUDACodegen().emit(
        subgraph_nodes, external_inputs, external_outputs)

``source`` is a kernel *body* for :func:`phew_b200.mx.fast.cuda_kernel` (the
``mx.fast.metal_kernel`` analogue), which wraps it in an ``extern "C"``
signature built from ``input_names`` / ``output_names`` and the dtypes of
the arrays it is called with.

Semantics (what the kernel computes) follow the reference emitter and the
MLX evaluation of the unfused graph:

* every node's result is rounded to that node's dtype, as the MSL kernel
  does by holding each value in a variable of the node's type
  (``msl_codegen.py:184-199``) and as MLX does between separate ops;
* add / sub / mul / div / sqrt use the IEEE round-to-nearest intrinsics
  (``__fadd_rn`` ...), so no multiply-add contraction changes a result;
* constants are inlined, rounded to their node's dtype
  (``msl_codegen.py:55-67, 189-191``);
* broadcast inputs are indexed from the flat output index
  (``msl_codegen.py:70-107``).

Layout and launch (the B200 part): the body is a grid-stride loop that moves
one 16-byte vector per array per iteration (8 x 16-bit or 4 x 32-bit
elements), with row-broadcast inputs (``elem % inner``) read as vectors too
and column-broadcast ones read once per vector.  Chains whose arrays are all
of one 16-bit float type compute in packed pairs (``add.rn.f16x2`` ...),
which give the same bits as fp32-then-round for add/sub/mul.  A scalar loop
handles the tail, unaligned pointers and general broadcasts.

Nodes are read by duck typing: the class name (or a ``kind`` attribute)
selects Elementwise / Cast / Constant, and the fields used are ``id``,
``shape``, ``dtype`` (an enum with ``.value`` or a plain string),
``inputs``, ``op``, ``value`` and ``target_dtype`` -- the fields of
``phew.ir.ops`` (``ir/ops.py:28-64,82-86``).
"""

from __future__ import annotations

import math
import struct
from typing import Any, Iterable

import numpy as np

try:  # bf16 rounding of constants
    import ml_dtypes as _mld
except ImportError:  # pragma: no cover - ml_dtypes ships with the image
    _mld = None

# ---------------------------------------------------------------------------
# dtype tables
# ---------------------------------------------------------------------------

FLOAT_TYPES = ("float32", "float16", "bfloat16")
HALF_TYPES = ("float16", "bfloat16")

CTYPE = {
    "float32": "float",
    "float16": "phew_f16",
    "bfloat16": "phew_bf16",
    "int8": "signed char",
    "int16": "short",
    "int32": "int",
    "int64": "long long",
    "uint8": "unsigned char",
    "uint16": "unsigned short",
    "uint32": "unsigned int",
    "uint64": "unsigned long long",
    "bool": "bool",
}

ITEMSIZE = {
    "float32": 4,
    "float16": 2,
    "bfloat16": 2,
    "int8": 1,
    "int16": 2,
    "int32": 4,
    "int64": 8,
    "uint8": 1,
    "uint16": 2,
    "uint32": 4,
    "uint64": 8,
    "bool": 1,
}

# Value type that holds a node's result inside the kernel.
VALUE_CTYPE = dict(CTYPE, float16="float", bfloat16="float")


def dtype_name(d: Any) -> str:
    """Normalise a dtype (phew Dtype enum, our mx Dtype, numpy dtype, str)."""
    if d is None:
        return "float32"
    for attr in ("value", "name"):
        v = getattr(d, attr, None)
        if isinstance(v, str):
            d = v
            break
    d = str(d)
    if d in ("bool_", "bool"):
        return "bool"
    return d


def node_kind(node: Any) -> str:
    return getattr(node, "kind", None) or type(node).__name__


def _numel(shape: Iterable[int]) -> int:
    n = 1
    for s in shape:
        n *= int(s)
    return n


# ---------------------------------------------------------------------------
# literals
# ---------------------------------------------------------------------------


def _round_value(value: float, dt: str) -> float:
    """Round a Python float the way an inlined literal of dtype `dt` is."""
    f = float(np.float32(value))
    if dt == "float16":
        return float(np.float16(f))
    if dt == "bfloat16":
        if _mld is None:
            raise ValueError("bfloat16 constants need ml_dtypes")
        return float(np.asarray(f, dtype=np.float32).astype(_mld.bfloat16).astype(np.float32))
    return f


def float_literal(value: float) -> str:
    """An exact fp32 C literal for `value` (already representable in fp32)."""
    f = float(np.float32(value))
    if math.isnan(f):
        return "__int_as_float(0x7fc00000)"
    if math.isinf(f):
        return "__int_as_float(0x7f800000)" if f > 0 else "__int_as_float(0xff800000)"
    bits = struct.unpack("<I", struct.pack("<f", f))[0]
    return f"__int_as_float(0x{bits:08x}) /* {f!r} */"


def half_bits(value: float, dt: str) -> int:
    """Raw 16-bit pattern of `value` rounded to dtype `dt`."""
    v = _round_value(value, dt)
    if dt == "float16":
        return int(np.asarray(v, dtype=np.float16).view(np.uint16))
    return int(np.asarray(v, dtype=np.float32).view(np.uint32)) >> 16


def _const_literal(value: Any, dt: str) -> str:
    if isinstance(value, (list, tuple, np.ndarray)) and np.ndim(value) > 0:
        raise ValueError("cuda_codegen: non-scalar Constant cannot be inlined")
    if dt in FLOAT_TYPES:
        return float_literal(_round_value(float(value), dt))
    if dt == "bool":
        return "true" if bool(value) else "false"
    iv = int(value)
    if dt in ("int64",):
        return f"{iv}LL"
    if dt in ("uint64",):
        return f"{iv}ULL"
    if dt.startswith("uint"):
        return f"{iv}u"
    return str(iv)


# ---------------------------------------------------------------------------
# op table: expression builders in the fp32 value domain
# ---------------------------------------------------------------------------

ALIASES = {
    "multiply": "mul",
    "subtract": "sub",
    "divide": "div",
    "neg": "negative",
    "equal": "eq",
    "not_equal": "ne",
    "greater": "gt",
    "greater_equal": "ge",
    "less": "lt",
    "less_equal": "le",
    "pow": "power",
    "atan2": "arctan2",
}

_UNARY_F = {
    "abs": "fabsf({a})",
    "log": "logf({a})",
    "sqrt": "__fsqrt_rn({a})",
    "rsqrt": "__fdiv_rn(1.0f, __fsqrt_rn({a}))",
    "relu": "phew_maximum({a}, 0.0f)",
    "gelu": "__fmul_rn(__fmul_rn({a}, 0.5f), __fadd_rn(1.0f, erff(__fmul_rn({a}, 0.70710678118654752f))))",
    "cos": "cosf({a})",
    "sin": "sinf({a})",
    "tan": "tanf({a})",
    "arctan": "atanf({a})",
    "arcsin": "asinf({a})",
    "arccos": "acosf({a})",
    "arctanh": "atanhf({a})",
    "arcsinh": "asinhf({a})",
    "arccosh": "acoshf({a})",
    "cosh": "coshf({a})",
    "sinh": "sinhf({a})",
    "degrees": "__fmul_rn({a}, 57.295779513082320876f)",
    "radians": "__fmul_rn({a}, 0.017453292519943295769f)",
    "square": "__fmul_rn({a}, {a})",
    "ceil": "ceilf({a})",
    "floor": "floorf({a})",
    "round": "rintf({a})",
    "sign": "phew_sign({a})",
    "reciprocal": "__fdiv_rn(1.0f, {a})",
    "erf": "erff({a})",
    "erfinv": "erfinvf({a})",
    "expm1": "expm1f({a})",
    "log1p": "log1pf({a})",
    "log2": "log2f({a})",
    "log10": "log10f({a})",
    "negative": "(-{a})",
}

# Transcendentals with a 16-bit-precision variant (used when the node's dtype
# is float16/bfloat16, whose result is rounded to 11/8 significant bits).
_UNARY_F_PRECISE = {
    "exp": "expf({a})",
    "sigmoid": "__fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-({a}))))",
    "tanh": "tanhf({a})",
    "silu": "__fdiv_rn({a}, __fadd_rn(1.0f, expf(-({a}))))",
}
_UNARY_F_HALF = {
    "exp": "phew_exp16({a})",
    "sigmoid": "phew_sigmoid16({a})",
    "tanh": "phew_tanh16({a})",
    "silu": "__fmul_rn({a}, phew_sigmoid16({a}))",
}
# Same ops at about 2^-20 relative error (twice the transcendental-unit work).
_UNARY_F_HALF_PRECISE = {
    "exp": "phew_exp16({a})",
    "sigmoid": "phew_sigmoid16p({a})",
    "tanh": "phew_tanh16p({a})",
    "silu": "__fmul_rn({a}, phew_sigmoid16p({a}))",
}

_BINARY_F = {
    "add": "__fadd_rn({a}, {b})",
    "sub": "__fsub_rn({a}, {b})",
    "mul": "__fmul_rn({a}, {b})",
    "div": "__fdiv_rn({a}, {b})",
    "maximum": "phew_maximum({a}, {b})",
    "minimum": "phew_minimum({a}, {b})",
    "logaddexp": "phew_logaddexp({a}, {b})",
    "floor_divide": "floorf(__fdiv_rn({a}, {b}))",
    "remainder": "phew_remainder({a}, {b})",
    "power": "powf({a}, {b})",
    "arctan2": "atan2f({a}, {b})",
}

_COMPARE = {"eq": "==", "ne": "!=", "gt": ">", "ge": ">=", "lt": "<", "le": "<="}
_LOGICAL = {"logical_and": "&&", "logical_or": "||"}

_INT_BINARY = {"add": "+", "sub": "-", "mul": "*"}

# Bool-valued tests of a float (NaN / infinity classification).
_PREDICATE = {
    "isnan": "isnan({a})",
    "isinf": "isinf({a})",
    "isfinite": "isfinite({a})",
    "isposinf": "({a} == __int_as_float(0x7f800000))",
    "isneginf": "({a} == __int_as_float(0xff800000u))",
}
# Integer / bool bit operations.
_BITWISE = {"bitwise_and": "&", "bitwise_or": "|", "bitwise_xor": "^", "left_shift": "<<",
            "right_shift": ">>"}

SUPPORTED_OPS = (
    set(_UNARY_F)
    | set(_UNARY_F_PRECISE)
    | set(_BINARY_F)
    | set(_COMPARE)
    | set(_LOGICAL)
    | {"logical_not", "where", "bitwise_invert"}
    | set(_PREDICATE)
    | set(_BITWISE)
    | set(ALIASES)
)

# Ops computed natively on packed 16-bit pairs.
_PACKED_NATIVE = {"add": "add", "sub": "sub", "mul": "mul", "square": "sq", "negative": "neg", "abs": "abs"}


def canonical_op(op: str) -> str:
    return ALIASES.get(op, op)


def _round_expr(expr: str, dt: str) -> str:
    if dt == "float16":
        return f"phew_rnd_f16({expr})"
    if dt == "bfloat16":
        return f"phew_rnd_bf16({expr})"
    return expr


def _to_float(v: str, dt: str) -> str:
    return v if dt in FLOAT_TYPES else f"(float)({v})"


def scalar_expr(
    op: str, args: list[str], arg_dtypes: list[str], out_dt: str, round_result: bool = True,
    precise16: bool = False,
) -> str:
    """C expression computing `op` on value variables, typed for `out_dt`.

    Float results are rounded to `out_dt` (unless `round_result` is False,
    for callers that round while packing); integer and bool results use C
    semantics of the node's C type.  `precise16` selects the slower,
    near-correctly-rounded tanh/sigmoid for 16-bit nodes.
    """
    op = canonical_op(op)
    if out_dt in FLOAT_TYPES:
        fa = [_to_float(a, d) for a, d in zip(args, arg_dtypes)]
        half = out_dt in HALF_TYPES
        if op in _COMPARE:
            expr = f"(({fa[0]} {_COMPARE[op]} {fa[1]}) ? 1.0f : 0.0f)"
        elif op in _LOGICAL:
            expr = f"(((({fa[0]}) != 0.0f) {_LOGICAL[op]} (({fa[1]}) != 0.0f)) ? 1.0f : 0.0f)"
        elif op == "logical_not":
            expr = f"(({fa[0]}) == 0.0f ? 1.0f : 0.0f)"
        elif op == "where":
            cond = args[0] if arg_dtypes[0] == "bool" else f"({fa[0]} != 0.0f)"
            expr = f"({cond} ? {fa[1]} : {fa[2]})"
        elif op in _UNARY_F and len(fa) >= 1:
            expr = _UNARY_F[op].format(a=fa[0])
        elif op in _UNARY_F_PRECISE and len(fa) >= 1:
            if half:
                table = _UNARY_F_HALF_PRECISE if precise16 else _UNARY_F_HALF
            else:
                table = _UNARY_F_PRECISE
            expr = table[op].format(a=fa[0])
        elif op in _BINARY_F and len(fa) == 2:
            expr = _BINARY_F[op].format(a=fa[0], b=fa[1])
        else:
            raise ValueError(f"cuda_codegen: unhandled op {op!r}")
        return _round_expr(expr, out_dt) if round_result else expr
    ct = VALUE_CTYPE[out_dt]
    if op in _COMPARE:
        return f"(({ct})({args[0]} {_COMPARE[op]} {args[1]}))"
    if op in _LOGICAL:
        return f"(({ct})({args[0]} {_LOGICAL[op]} {args[1]}))"
    if op == "logical_not":
        return f"(({ct})(!{args[0]}))"
    if op == "where":
        return f"(({ct})({args[0]} ? {args[1]} : {args[2]}))"
    if op in _PREDICATE:
        return f"(({ct}){_PREDICATE[op].format(a=_to_float(args[0], arg_dtypes[0]))})"
    if op in _BITWISE:
        if arg_dtypes[0] in FLOAT_TYPES or arg_dtypes[1] in FLOAT_TYPES:
            raise ValueError(f"cuda_codegen: {op} of floating-point values")
        return f"(({ct})({args[0]} {_BITWISE[op]} {args[1]}))"
    if op == "bitwise_invert":
        if arg_dtypes[0] in FLOAT_TYPES:
            raise ValueError("cuda_codegen: bitwise_invert of floating-point values")
        return f"(({ct})(!{args[0]}))" if out_dt == "bool" else f"(({ct})(~{args[0]}))"
    if out_dt == "bool":
        raise ValueError(f"cuda_codegen: unhandled bool op {op!r}")
    if op in _INT_BINARY and len(args) == 2:
        return f"(({ct})({args[0]} {_INT_BINARY[op]} {args[1]}))"
    if op == "negative":
        return f"(({ct})(-{args[0]}))"
    if op == "abs":
        return f"(({ct})({args[0]} < 0 ? -{args[0]} : {args[0]}))"
    if op == "square":
        return f"(({ct})({args[0]} * {args[0]}))"
    if op == "maximum":
        return f"(({ct})({args[0]} > {args[1]} ? {args[0]} : {args[1]}))"
    if op == "minimum":
        return f"(({ct})({args[0]} < {args[1]} ? {args[0]} : {args[1]}))"
    if op == "floor_divide":
        return f"phew_floordiv_i({args[0]}, {args[1]})"
    if op == "remainder":
        return f"phew_remainder_i({args[0]}, {args[1]})"
    if op == "sign":
        return f"(({ct})(({args[0]} > 0) - ({args[0]} < 0)))"
    raise ValueError(f"cuda_codegen: unhandled integer op {op!r}")


def cast_expr(v: str, src_dt: str, dst_dt: str) -> str:
    """Value-domain conversion for a Cast node (MLX astype semantics)."""
    if dst_dt in FLOAT_TYPES:
        return _round_expr(_to_float(v, src_dt), dst_dt)
    ct = VALUE_CTYPE[dst_dt]
    if dst_dt == "bool":
        return f"({v} != 0)"
    if src_dt in FLOAT_TYPES:
        return f"(({ct})truncf({v}))"
    return f"(({ct})({v}))"


# ---------------------------------------------------------------------------
# broadcast classification
# ---------------------------------------------------------------------------


def broadcast_compatible(in_shape, out_shape) -> bool:
    if len(in_shape) > len(out_shape):
        return False
    padded = (1,) * (len(out_shape) - len(in_shape)) + tuple(in_shape)
    return all(i == 1 or i == o for i, o in zip(padded, out_shape))


def classify_input(in_shape, out_shape) -> tuple[str, int]:
    """Return (class, extent) of an input's broadcast pattern.

    classes: "full" (same shape), "scalar" (one element), "suffix" (equals
    the trailing dims: index ``elem % extent``), "prefix" (equals the leading
    dims: index ``elem / extent``) and "general" (anything else).
    """
    in_shape = tuple(int(s) for s in in_shape)
    out_shape = tuple(int(s) for s in out_shape)
    if in_shape == out_shape:
        return "full", 0
    if _numel(in_shape) == 1:
        return "scalar", 0
    nd = len(out_shape)
    padded = (1,) * (nd - len(in_shape)) + in_shape
    for k in range(nd + 1):
        if all(p == 1 for p in padded[:k]) and padded[k:] == out_shape[k:]:
            return "suffix", _numel(out_shape[k:])
    for k in range(nd + 1):
        if padded[:k] == out_shape[:k] and all(p == 1 for p in padded[k:]):
            return "prefix", _numel(out_shape[k:])
    return "general", 0


IO_TAG = "// phew-io:"


# A broadcast input below this size stays in the L2 (126 MB on B200) between
# the row groups that re-read it, so its rows need no reordering.
SHARED_ROWS_MIN_BYTES = 16 << 20


def shared_row_groups(classes, out_shape, itemsizes) -> tuple[int, int] | None:
    """(outer, inner) when a "suffix" input of at least SHARED_ROWS_MIN_BYTES
    spans several rows of the output (an additive mask (L, L) under scores
    (B, H, L, L)): the output's ``outer * inner`` rows fall into `outer`
    groups of `inner` rows that read the same `inner` rows of that input.
    None when no input does."""
    cols = int(out_shape[-1])
    n = _numel(out_shape)
    ext = max([e for (c, e), size in zip(classes, itemsizes)
               if c == "suffix" and e > cols and n % e == 0 and e * size >= SHARED_ROWS_MIN_BYTES]
              or [0])
    if not ext or n == ext:
        return None
    return n // ext, ext // cols


def io_contract_line(classes, out_shape, in_shapes, it: str) -> str:
    """Machine-readable launch contract checked by the kernel factory before
    every launch, so a body specialised to traced shapes can never index
    outside the arrays it is given (see ``kernel.check_io_contract``)."""
    parts = ["idx32" if it == "unsigned int" else "idx64"]
    parts.append("out=" + "x".join(str(int(s)) for s in out_shape))
    for k, ((cls, ext), shp) in enumerate(zip(classes, in_shapes)):
        if cls in ("suffix", "prefix"):
            parts.append(f"inp{k}={cls}:{ext}")
        elif cls == "general":
            parts.append(f"inp{k}=general:" + "x".join(str(int(s)) for s in shp))
        else:
            parts.append(f"inp{k}={cls}")
    return IO_TAG + " " + " ".join(parts)


def general_index(elem: str, out_shape, in_shape, it: str) -> str:
    """Flat input index of a general broadcast (restates msl_codegen.py:70-107)."""
    ndim = len(out_shape)
    padded = (1,) * (ndim - len(in_shape)) + tuple(in_shape)
    out_strides, s = [], 1
    for d in reversed(out_shape):
        out_strides.insert(0, s)
        s *= d
    in_strides, s = [], 1
    for d in reversed(padded):
        in_strides.insert(0, s)
        s *= d
    terms = []
    u = "u" if it == "unsigned int" else "ull"
    for i in range(ndim):
        if padded[i] == 1:
            continue
        coord = (
            f"({elem} % {out_shape[i]}{u})"
            if out_strides[i] == 1
            else f"(({elem} / {out_strides[i]}{u}) % {out_shape[i]}{u})"
        )
        terms.append(coord if in_strides[i] == 1 else f"{coord} * {in_strides[i]}{u}")
    return " + ".join(terms) if terms else "0"


# ---------------------------------------------------------------------------
# emitter
# ---------------------------------------------------------------------------


class SubgraphCUDACodegen:
    """Emit a CUDA kernel body for a fuseable subgraph.

    Parameters of :meth:`emit` mirror ``SubgraphMSLCodegen.emit``:
    topologically ordered Elementwise/Cast/Constant nodes, the external
    input nodes (become ``inp0, inp1, ...``) and the external output nodes
    (become ``out0, out1, ...``).  Raises ``ValueError`` for anything it
    cannot fuse; the fusion pass treats that as "leave the chain unfused"
    (``rules/fusion.py:266-270``).

    ``precise_16bit=True`` computes tanh / sigmoid / silu of 16-bit nodes
    with about 2^-20 relative error instead of the hardware tanh
    approximation (about 2^-11, at most a couple of ulps of the 16-bit
    result); it costs twice the transcendental-unit throughput, which bounds
    the benchmark chain.
    """

    def __init__(self, precise_16bit: bool = False) -> None:
        self.precise_16bit = precise_16bit

    def emit(
        self,
        subgraph_nodes: list[Any],
        external_inputs: list[Any],
        external_outputs: list[Any],
    ) -> tuple[str, list[str], list[str]]:
        if not external_outputs:
            raise ValueError("cuda_codegen: chain has no external output")
        inp_names = [f"inp{i}" for i in range(len(external_inputs))]
        out_names = [f"out{i}" for i in range(len(external_outputs))]
        out_shape = tuple(int(s) for s in external_outputs[0].shape)
        n = _numel(out_shape)
        for o in external_outputs:
            if tuple(int(s) for s in o.shape) != out_shape:
                raise ValueError(
                    "cuda_codegen: external outputs of different shapes cannot share one "
                    "iteration space"
                )
        in_dts = [dtype_name(x.dtype) for x in external_inputs]
        out_dts = [dtype_name(x.dtype) for x in external_outputs]
        for d in in_dts + out_dts:
            if d not in CTYPE:
                raise ValueError(f"cuda_codegen: unsupported dtype {d!r}")
        classes = []
        for x in external_inputs:
            shp = tuple(int(s) for s in x.shape)
            if len(shp) > 0 and not broadcast_compatible(shp, out_shape):
                raise ValueError("cuda_codegen: input not broadcast-compatible with output")
            classes.append(classify_input(shp, out_shape))

        # Resolve the chain into a statement plan (also validates every op).
        plan = _Plan(subgraph_nodes, external_inputs, external_outputs,
                     precise16=getattr(self, "precise_16bit", False))

        # 32-bit indexing when the traced size leaves 2x headroom; the runtime
        # factory refuses launches whose size would overflow it.
        it = "unsigned int" if n < 2**30 else "unsigned long long"
        u = "u" if it == "unsigned int" else "ull"
        itemsizes = [ITEMSIZE[d] for d, (c, _) in zip(in_dts, classes) if c in ("full", "suffix")]
        itemsizes += [ITEMSIZE[d] for d in out_dts]
        V = max(1, min(8, 16 // min(itemsizes)))
        half_t = plan.pure_half_type(in_dts, out_dts)
        vec_ok_classes = all(
            c in ("full", "scalar", "general")
            or (c == "suffix" and ext % V == 0)
            or (c == "prefix" and ext % V == 0)
            for c, ext in classes
        )

        L: list[str] = []
        L.append(
            f"// fused elementwise chain: {len(plan.compute_nodes)} ops, "
            f"{len(external_inputs)} inputs, {len(external_outputs)} outputs, {n} elements"
        )
        L.append(io_contract_line(classes, out_shape, [tuple(x.shape) for x in external_inputs], it))
        # The element count comes from the launch (the output's size), so the
        # kernel traced at one size also runs the other verification sizes.
        L.append(f"const {it} phew_n = ({it}){out_names[0]}_size;")
        L.append(f"const {it} phew_tid = ({it})blockIdx.x * blockDim.x + threadIdx.x;")
        L.append(f"const {it} phew_nthreads = ({it})gridDim.x * blockDim.x;")
        L.append(f"{it} phew_tail = 0;")
        # Loop-invariant constants.
        for line in plan.constant_lines(packed_type=half_t if (vec_ok_classes and V == 8) else None):
            L.append(line)

        if vec_ok_classes and n >= V:
            ptrs = " | ".join(f"reinterpret_cast<phew_uptr>({nm})" for nm in inp_names + out_names)
            L.append(f"if ((({ptrs}) & 15u) == 0u) {{")
            L.append(f"  const {it} phew_nvec = phew_n / {V}{u};")
            L.append(
                f"  for ({it} phew_v = phew_tid; phew_v < phew_nvec; phew_v += phew_nthreads) {{"
            )
            L.append(f"    const {it} elem = phew_v * {V}{u};")
            body = self._vector_body(
                plan, external_inputs, inp_names, out_names, in_dts, out_dts, classes,
                out_shape, V, it, u, half_t,
            )
            L.extend("    " + b for b in body)
            L.append("  }")
            L.append(f"  phew_tail = phew_nvec * {V}{u};")
            L.append("}")

        L.append(f"for ({it} elem = phew_tail + phew_tid; elem < phew_n; elem += phew_nthreads) {{")
        scalar = self._scalar_body(
            plan, external_inputs, inp_names, out_names, in_dts, out_dts, classes, out_shape, it, u
        )
        L.extend("  " + s for s in scalar)
        L.append("}")
        source = "\n".join(f"    {line}" if line else "" for line in L)
        return source, inp_names, out_names

    # -- elementwise prologue fused into a row softmax --------------------------

    def emit_softmax(self, subgraph_nodes, external_inputs, root, tpr: int, rpb: int,
                     vpt: int) -> tuple[str, list[str], list[str]]:
        """Body of ``softmax(root, axis=-1)`` where `root` is the value of the
        elementwise DAG `subgraph_nodes` over `external_inputs`: each row's
        elements are computed in registers (rounded per node, as the chain
        kernels round them) and never written to HBM.

        The thread/element mapping and both reductions are those of
        ``csrc/rows.cu``'s ``softmax_vec_kernel`` for the same row plan (`tpr`
        threads per row, `rpb` rows per block, `vpt` 16-byte vectors per
        thread), so the result has the bits of materialising `root` and then
        calling ``phew_softmax``.  Launch: block (tpr, rpb), one block per
        `rpb` rows.  Raises ``ValueError`` when the DAG cannot run 16 bytes
        at a time in that mapping (the caller then materialises `root`).
        """
        out_shape = tuple(int(x) for x in root.shape)
        if not out_shape:
            raise ValueError("cuda_codegen: softmax of a 0-d array")
        cols = out_shape[-1]
        out_dt = dtype_name(root.dtype)
        if out_dt not in ("float32", "float16", "bfloat16"):
            raise ValueError(f"cuda_codegen: softmax over {out_dt}")
        E = 16 // ITEMSIZE[out_dt]
        if cols % E:
            raise ValueError("cuda_codegen: softmax row is not a whole number of vectors")
        in_dts = [dtype_name(x.dtype) for x in external_inputs]
        for d in in_dts:
            if d not in CTYPE:
                raise ValueError(f"cuda_codegen: unsupported dtype {d!r}")
        classes = []
        for x in external_inputs:
            shp = tuple(int(v) for v in x.shape)
            if len(shp) > 0 and not broadcast_compatible(shp, out_shape):
                raise ValueError("cuda_codegen: input not broadcast-compatible with output")
            classes.append(classify_input(shp, out_shape))
        itemsizes = [ITEMSIZE[d] for d, (c, _) in zip(in_dts, classes) if c in ("full", "suffix")]
        V = max(1, min(8, 16 // min(itemsizes + [ITEMSIZE[out_dt]])))
        if V != E:
            raise ValueError("cuda_codegen: input vectors narrower than the softmax rows'")
        if not all(c in ("full", "scalar", "general") or ext % V == 0 for c, ext in classes):
            raise ValueError("cuda_codegen: broadcast extent not a multiple of the vector")
        plan = _Plan(subgraph_nodes, external_inputs, [root],
                     precise16=getattr(self, "precise_16bit", False))
        inp_names = [f"inp{i}" for i in range(len(external_inputs))]
        out_names = ["out0"]
        n = _numel(out_shape)
        it = "unsigned int" if n < 2**30 else "unsigned long long"
        u = "u" if it == "unsigned int" else "ull"
        half_t = plan.pure_half_type(in_dts, [out_dt])
        packed = half_t is not None and V == 8
        body = self._vector_body(plan, external_inputs, inp_names, out_names, in_dts, [out_dt],
                                 classes, out_shape, V, it, u, half_t)
        body = [b for b in body if not b.startswith("phew_stv<")]
        ct = CTYPE[out_dt]
        st = f"phew_st_{_suffix(out_dt)}"
        div = "__fdiv_rn(phew_sv[j][l], phew_s)" if out_dt == "float32" else "phew_sv[j][l] * phew_inv"
        # Rows that share a large broadcast input's rows run next to one
        # another: position p takes row (p % outer) * inner + p / outer, so
        # the `outer` readers of one mask row are in flight together and that
        # row is read from HBM once instead of once per head (a seq-8192
        # mask is 134 MB, more than the L2).  Only which block takes which row
        # changes, not any row's arithmetic.
        groups = shared_row_groups(classes, out_shape, [ITEMSIZE[d] for d in in_dts])
        rows = n // cols
        # When the plan covers a row exactly (tpr * vpt vectors), no load
        # needs a guard: a spare row of the last block reads the last row and
        # stores nothing.  The kernel is then straight-line code, which keeps
        # all of a thread's loads in flight at once (the guarded form ran a
        # seq-8192 score softmax at 0.71 of the HBM copy rate, the unguarded
        # one at 0.96, same bits).
        exact = tpr * vpt == cols // V
        contract = io_contract_line(classes, out_shape, [tuple(x.shape) for x in external_inputs], it)
        contract += f" rowlen={cols}"
        row_lines = [f"const {it} phew_pos = ({it})blockIdx.x * blockDim.y + threadIdx.y;",
                     "const bool phew_active = phew_pos < phew_rows;"]
        if exact:
            # the launch is block (tpr, rpb); spare rows take the last row
            row_lines += [f"if (blockDim.x != {tpr}u || blockDim.y != {rpb}u) return;",
                          f"const {it} phew_p = phew_active ? phew_pos : phew_rows - 1{u};"]
        else:
            row_lines += [f"const {it} phew_p = phew_pos;"]
        if groups is None:
            row_lines += [f"const {it} phew_row = phew_p;"]
        else:
            outer, inner = groups
            contract += f" rows={rows}"
            row_lines += [f"const {it} phew_row = (phew_p % {outer}{u}) * {inner}{u} + phew_p / {outer}{u};"]
        if exact:
            guard, store_guard = "true", "true"
            vi = f"threadIdx.x + ({it})j * {tpr}{u}"
        else:
            guard, store_guard = "phew_active && phew_vi < phew_nvec", "phew_vi < phew_nvec"
            vi = f"threadIdx.x + ({it})j * blockDim.x"
        L: list[str] = []
        L.append(
            f"// elementwise prologue ({len(plan.compute_nodes)} ops, {len(external_inputs)} inputs) "
            f"+ softmax over rows of {cols}"
        )
        L.append(contract)
        for line in plan.constant_lines(packed_type=half_t if packed else None):
            L.append(line)
        L += [
            "__shared__ float phew_smem[32 * 32];",
            f"const {it} phew_cols = {cols}{u};",
            f"const {it} phew_rows = ({it})out0_size / phew_cols;",
            f"const {it} phew_nvec = phew_cols / {V}{u};",
            *row_lines,
            f"float phew_sv[{vpt}][{V}];",
            "float phew_m = __int_as_float(0xff800000u);",
            "#pragma unroll",
            f"for (int j = 0; j < {vpt}; ++j) {{",
            f"  const {it} phew_vi = {vi};",
            f"  if ({guard}) {{",
            f"    const {it} elem = phew_row * phew_cols + phew_vi * {V}{u};",
        ]
        L += ["    " + b for b in body]
        L += [
            "    #pragma unroll",
            f"    for (int l = 0; l < {V}; ++l) phew_sv[j][l] = phew_ld(st0.v[l]);",
            "    #pragma unroll",
            f"    for (int l = 0; l < {V}; ++l) phew_m = fmaxf(phew_m, phew_sv[j][l]);",
            "  }",
            "}",
            "phew_m = phew_row_allreduce<true>(phew_m, phew_smem);",
            "float phew_s = 0.f;",
            "#pragma unroll",
            f"for (int j = 0; j < {vpt}; ++j) {{",
            f"  const {it} phew_vi = {vi};",
            f"  if ({guard}) {{",
            "    #pragma unroll",
            f"    for (int l = 0; l < {V}; ++l) {{",
            f"      phew_sv[j][l] = phew_softmax_exp<{ITEMSIZE[out_dt]}>(phew_sv[j][l] - phew_m);",
            "      phew_s += phew_sv[j][l];",
            "    }",
            "  }",
            "}",
            "phew_s = phew_row_allreduce<false>(phew_s, phew_smem);",
            "if (!phew_active) return;",
            "const float phew_inv = 1.0f / phew_s;",
            "#pragma unroll",
            f"for (int j = 0; j < {vpt}; ++j) {{",
            f"  const {it} phew_vi = {vi};",
            f"  if ({store_guard}) {{",
            f"    phew_vec<{ct}, {V}> phew_o;",
            "    #pragma unroll",
            f"    for (int l = 0; l < {V}; ++l) phew_o.v[l] = {st}({div});",
            f"    phew_stv<{ct}, {V}>(out0 + phew_row * phew_cols + phew_vi * {V}{u}, phew_o);",
            "  }",
            "}",
        ]
        _ = packed
        source = "\n".join(f"    {line}" if line else "" for line in L)
        return source, inp_names, out_names

    # -- elementwise prologue fused into a row reduction ------------------------

    ROW_STAGE_BYTES = 32 * 1024  # static shared memory for a row map's staged input rows (both buffers)

    _REDUCE_INIT = {"sum": "0.0f", "mean": "0.0f", "prod": "1.0f",
                    "max": "__int_as_float(0xff800000u)", "min": "__int_as_float(0x7f800000u)"}

    def emit_reduce_rows(self, subgraph_nodes, external_inputs, root, op: str, keepdims: bool,
                         tpr: int, rpb: int) -> tuple[str, list[str], list[str]]:
        """Body of ``op(root, axis=-1)`` (sum / mean / max / min / prod) where
        `root` is the value of the elementwise DAG `subgraph_nodes`: each
        element is computed (rounded per node) as the reduction reads it and
        never written to HBM.  Thread mapping, accumulation order and the
        shuffle / shared-memory tree are those of ``csrc/rows.cu``'s
        ``reduce_rows_kernel`` (`tpr` threads per row striding over it, `rpb`
        rows per block), so the result has the bits of materialising `root`
        and then calling ``phew_reduce``.  Raises ``ValueError`` when it
        cannot (the caller then materialises `root`)."""
        out_shape = tuple(int(x) for x in root.shape)
        if not out_shape or op not in self._REDUCE_INIT:
            raise ValueError("cuda_codegen: not a row reduction")
        red = out_shape[-1]
        out_dt = dtype_name(root.dtype)
        if out_dt not in ("float32", "float16", "bfloat16"):
            raise ValueError(f"cuda_codegen: reduction over {out_dt}")
        in_dts = [dtype_name(x.dtype) for x in external_inputs]
        classes = []
        for x in external_inputs:
            shp = tuple(int(v) for v in x.shape)
            if len(shp) > 0 and not broadcast_compatible(shp, out_shape):
                raise ValueError("cuda_codegen: input not broadcast-compatible with output")
            cls = classify_input(shp, out_shape)
            if cls[0] == "general":
                raise ValueError("cuda_codegen: general broadcast in a fused reduction")
            classes.append(cls)
        plan = _Plan(subgraph_nodes, external_inputs, [root],
                     precise16=getattr(self, "precise_16bit", False))
        inp_names = [f"inp{i}" for i in range(len(external_inputs))]
        n = _numel(out_shape)
        it = "unsigned int" if n < 2**30 else "unsigned long long"
        u = "u" if it == "unsigned int" else "ull"
        L: list[str] = []
        L.append(f"// elementwise prologue ({len(plan.compute_nodes)} ops) + {op} over rows of {red}")
        L.append(io_contract_line(classes, out_shape, [tuple(x.shape) for x in external_inputs], it)
                 + f" rowred={red}")
        L += plan.constant_lines(packed_type=None)
        L.append("__shared__ float phew_smem[32 * 32];")
        L += self._row_reduce_lines(plan, external_inputs, inp_names, in_dts, classes, out_shape,
                                    op, f"({it})out0_size", it, u)
        L += [
            "if (phew_active && threadIdx.x == 0) {",
            ("  phew_acc = __fdiv_rn(phew_acc, (float)phew_red);" if op == "mean" else ""),
            f"  out0[phew_row] = phew_st_{_suffix(out_dt)}(phew_acc);",
            "}",
        ]
        _ = keepdims
        source = "\n".join(f"    {line}" if line else "" for line in L)
        return source, inp_names, ["out0"]

    def _row_reduce_lines(self, plan, ext_in, names, in_dts, classes, out_shape, op: str,
                          rows_expr: str, it: str, u: str, staged: dict | None = None,
                          after_header=(), header: bool = True) -> list[str]:
        """Rows of `out_shape[-1]` elements of `plan`'s single output, reduced
        with ``op`` into ``phew_acc`` (valid in every thread of the row after
        the code): `blockDim.x` threads per row, thread t accumulating
        elements t, t + blockDim.x, ... in order, then a butterfly over the
        warp and, across warps, over their partials in shared memory
        (``phew_smem``, declared by the caller).  The order of
        ``csrc/rows.cu``'s ``reduce_rows_kernel``.  Inputs named in `staged`
        are read from that shared-memory copy of the row (``phew_lrow`` is
        the row's offset in it); `after_header` lines go between the row
        bookkeeping and the accumulation."""
        red = out_shape[-1]
        staged = staged or {}
        env = {}
        body = []
        for node, nm, dt, (cls, ext) in zip(ext_in, names, in_dts, classes):
            v = plan.var(node)
            if nm in staged and cls == "full":
                src = f"{staged[nm]}[phew_lrow + phew_c]"
            else:
                src = f"{nm}[{self._index(cls, ext, nm, node, out_shape, it, u)}]"
            body.append(f"const {VALUE_CTYPE[dt]} {v} = phew_ld({src});")
            env[node.id] = (v, dt)
        body += plan.scalar_lines(env)
        rv, rdt = env[plan.outputs[0].id]
        if rdt != dtype_name(plan.outputs[0].dtype):
            raise ValueError("cuda_codegen: reduction dtype differs from its input's")
        if op in ("max", "min"):
            cmp = ">" if op == "max" else "<"
            comb = ("phew_acc = ((phew_x {c} phew_acc || isnan(phew_x)) && !isnan(phew_acc)) ? phew_x : phew_acc;"
                    .format(c=cmp))
        elif op == "prod":
            comb = "phew_acc = phew_acc * phew_x;"
        else:
            comb = "phew_acc = phew_acc + phew_x;"
        shfl_comb = comb.replace("phew_x", "phew_y")
        L = [
            f"const {it} phew_red = {red}{u};",
            f"const {it} phew_rows = {rows_expr};",
            f"const {it} phew_row = ({it})blockIdx.x * blockDim.y + threadIdx.y;",
            "const bool phew_active = phew_row < phew_rows;",
        ] if header else []
        L += [
            *after_header,
            f"float phew_acc = {self._REDUCE_INIT[op]};",
            "if (phew_active) {",
            f"  for ({it} phew_c = threadIdx.x; phew_c < phew_red; phew_c += blockDim.x) {{",
            f"    const {it} elem = phew_row * phew_red + phew_c;",
        ]
        L += ["    " + b for b in body]
        L += [
            f"    const float phew_x = {rv};",
            "    " + comb,
            "  }",
            "}",
            "#pragma unroll",
            "for (int phew_o = 16; phew_o > 0; phew_o >>= 1) {",
            "  const float phew_y = __shfl_xor_sync(0xffffffffu, phew_acc, phew_o);",
            "  " + shfl_comb,
            "}",
            "{",
            "  const int phew_wpr = blockDim.x / 32;",
            "  if (phew_wpr > 1) {",
            "    const int phew_lane = threadIdx.x & 31, phew_warp = threadIdx.x >> 5;",
            "    float* phew_rs = phew_smem + threadIdx.y * 32;",
            "    __syncthreads();",
            "    if (phew_lane == 0) phew_rs[phew_warp] = phew_acc;",
            "    __syncthreads();",
            f"    phew_acc = phew_lane < phew_wpr ? phew_rs[phew_lane] : {self._REDUCE_INIT[op]};",
            "    #pragma unroll",
            "    for (int phew_o = 16; phew_o > 0; phew_o >>= 1) {",
            "      const float phew_y = __shfl_xor_sync(0xffffffffu, phew_acc, phew_o);",
            "      " + shfl_comb,
            "    }",
            "  }",
            "}",
        ]
        return L

    # -- row reduction broadcast back into an elementwise chain ----------------

    def emit_row_map(self, reduce_nodes, reduce_ext, reduce_root, op: str, map_nodes, map_ext,
                     map_root, row_value, slots: dict, tpr: int, rpb: int
                     ) -> tuple[str, list[str], list[str]]:
        """Body of ``map_root`` where the elementwise DAG `map_nodes` reads
        `row_value` = ``op(reduce_root, axis=-1, keepdims=True)`` of the
        elementwise DAG `reduce_nodes` over the same rows (the
        ``x * x -> mean -> rsqrt(. + eps) * x * w`` shape of an RMS norm):
        one block row computes its row's reduction, then the mapped chain over
        the row, so the reduced value never goes through HBM.

        Bits: the reduction is ``_row_reduce_lines`` (the order of
        ``reduce_rows_kernel``); row thread 0's result is rounded to the
        reduction's dtype -- the value ``emit_reduce_rows`` would store --
        and handed to the row's threads through shared memory; the mapped
        chain then runs the per-element code of ``emit`` with that value in
        place of its load.  So the result has the bits of materialising the
        reduction and then the chain.

        `slots` maps the id of every external spec of both DAGs except
        `row_value` to its kernel input index.  Launch: block (tpr, rpb), any
        number of blocks (each walks groups of `rpb` rows with a grid
        stride).  Raises ``ValueError`` when it cannot."""
        out_shape = tuple(int(x) for x in map_root.shape)
        if not out_shape or op not in self._REDUCE_INIT:
            raise ValueError("cuda_codegen: not a row map")
        if tuple(int(x) for x in reduce_root.shape) != out_shape:
            raise ValueError("cuda_codegen: reduction rows differ from the mapped rows")
        if tuple(int(x) for x in row_value.shape) != out_shape[:-1] + (1,):
            raise ValueError("cuda_codegen: row value is not one per row")
        red = out_shape[-1]
        red_dt = dtype_name(reduce_root.dtype)
        out_dt = dtype_name(map_root.dtype)
        if red_dt not in ("float32", "float16", "bfloat16") or dtype_name(row_value.dtype) != red_dt:
            raise ValueError("cuda_codegen: row map over a non-float reduction")
        if out_dt not in CTYPE:
            raise ValueError(f"cuda_codegen: unsupported dtype {out_dt!r}")
        n_in = max(slots.values()) + 1 if slots else 0
        in_shape: list = [None] * n_in
        in_dt: list = [None] * n_in
        for x in list(reduce_ext) + [m for m in map_ext if m is not row_value]:
            k = slots[x.id]
            in_shape[k] = tuple(int(v) for v in x.shape)
            in_dt[k] = dtype_name(x.dtype)
        if any(s is None for s in in_shape):
            raise ValueError("cuda_codegen: unused kernel input slot")
        classes = []
        for shp in in_shape:
            if len(shp) > 0 and not broadcast_compatible(shp, out_shape):
                raise ValueError("cuda_codegen: input not broadcast-compatible with output")
            cls = classify_input(shp, out_shape)
            if cls[0] == "general":
                raise ValueError("cuda_codegen: general broadcast in a row map")
            classes.append(cls)
        for d in in_dt:
            if d not in CTYPE:
                raise ValueError(f"cuda_codegen: unsupported dtype {d!r}")
        names = [f"inp{k}" for k in range(n_in)]
        n = _numel(out_shape)
        it = "unsigned int" if n < 2**30 else "unsigned long long"
        u = "u" if it == "unsigned int" else "ull"
        precise = getattr(self, "precise_16bit", False)
        rplan = _Plan(reduce_nodes, reduce_ext, [reduce_root], precise16=precise)
        mplan = _Plan(map_nodes, map_ext, [map_root], precise16=precise, prefix="w")
        r_names = [names[slots[x.id]] for x in reduce_ext]
        r_dts = [in_dt[slots[x.id]] for x in reduce_ext]
        r_classes = [classes[slots[x.id]] for x in reduce_ext]

        # The mapped chain reads the row value as a one-element local array
        # (the "scalar" load form), every other input as the chain kernel does.
        m_names, m_dts, m_classes = [], [], []
        for x in map_ext:
            if x is row_value:
                m_names.append("phew_rowv")
                m_dts.append(red_dt)
                m_classes.append(("scalar", 1))
            else:
                m_names.append(names[slots[x.id]])
                m_dts.append(in_dt[slots[x.id]])
                m_classes.append(classes[slots[x.id]])
        itemsizes = [ITEMSIZE[d] for d, (c, _) in zip(m_dts, m_classes) if c in ("full", "suffix")]
        itemsizes.append(ITEMSIZE[out_dt])
        V = max(1, min(8, 16 // min(itemsizes)))
        half_t = mplan.pure_half_type(m_dts, [out_dt])
        vec_ok = red % V == 0 and all(c in ("full", "scalar") or ext % V == 0 for c, ext in m_classes)
        packed = vec_ok and half_t is not None and V == 8

        # Rows of the full-size inputs are staged in shared memory, double
        # buffered: each block walks row groups (rpb rows) with a grid
        # stride and copies the next group's rows in with cp.async while it
        # reduces and maps the current one, so loads stay in flight through
        # the whole kernel.  The reduction reads the staged rows in its
        # fixed (strided) order, the chain reads them again: one HBM pass.
        full = [k for k in range(n_in) if classes[k][0] == "full"]
        stage_bytes = 2 * rpb * red * sum(ITEMSIZE[in_dt[k]] for k in full)
        staged = ({names[k]: f"phew_stg{k}" for k in full}
                  if full and stage_bytes <= self.ROW_STAGE_BYTES else {})
        buf = rpb * red  # elements per buffer of one staged input

        L: list[str] = []
        L.append(f"// {op} over rows of {red} ({len(rplan.compute_nodes)}-op prologue), broadcast into "
                 f"a {len(mplan.compute_nodes)}-op chain over the same rows; persistent row groups")
        L.append(io_contract_line(classes, out_shape, in_shape, it) + f" rowlen={red}")
        L += rplan.constant_lines(packed_type=None)
        L += mplan.constant_lines(packed_type=half_t if packed else None)
        L.append("__shared__ float phew_smem[32 * 32];")
        L.append(f"__shared__ {CTYPE[red_dt]} phew_rowv_s[32];")
        for k in (full if staged else []):
            L.append(f"__shared__ __align__(16) {CTYPE[in_dt[k]]} phew_stg{k}[{2 * buf}];")
        L += [
            f"const {it} phew_red = {red}{u};",
            f"const {it} phew_rows = ({it})out0_size / {red}{u};",
            f"const {it} phew_groups = (phew_rows + blockDim.y - 1) / blockDim.y;",
            f"const {it} phew_lrow0 = ({it})threadIdx.y * phew_red;",
        ]
        if staged:
            L.append(f"auto phew_stage = [&]({it} phew_gs, int phew_bs) {{")
            L.append(f"  const {it} phew_rs = phew_gs * blockDim.y + threadIdx.y;")
            L.append("  if (phew_rs >= phew_rows) return;")
            for k in full:
                ct, isz = CTYPE[in_dt[k]], ITEMSIZE[in_dt[k]]
                E = 16 // isz
                L.append("  {")
                L.append(f"    const {ct}* phew_src = {names[k]} + phew_rs * phew_red;")
                L.append(f"    {ct}* phew_dst = phew_stg{k} + ({it})phew_bs * {buf}{u} + phew_lrow0;")
                if (red * isz) % 16 == 0:
                    L += [
                        "    if ((reinterpret_cast<phew_uptr>(phew_src) & 15u) == 0u) {",
                        f"      for ({it} phew_q = threadIdx.x; phew_q < {red // E}{u}; phew_q += blockDim.x)",
                        f"        phew_cp_async16(phew_dst + phew_q * {E}{u}, phew_src + phew_q * {E}{u});",
                        "    } else {",
                    ]
                else:
                    L.append("    {")
                L += [
                    f"      for ({it} phew_c = threadIdx.x; phew_c < phew_red; phew_c += blockDim.x)",
                    "        phew_dst[phew_c] = phew_src[phew_c];",
                    "    }",
                    "  }",
                ]
            L.append("};")
        L += [
            f"{it} phew_g = blockIdx.x;",
            "int phew_buf = 0;",
        ]
        if staged:
            L += ["if (phew_g < phew_groups) phew_stage(phew_g, 0);", "phew_cp_commit();"]
        L.append("for (; phew_g < phew_groups; phew_g += gridDim.x, phew_buf ^= 1) {")
        body_lines: list[str] = []
        if staged:
            body_lines += [
                "if (phew_g + gridDim.x < phew_groups) phew_stage(phew_g + gridDim.x, phew_buf ^ 1);",
                "phew_cp_commit();",
                "phew_cp_wait1();  // this group's rows have landed (the next group's may be in flight)",
                "__syncthreads();",
            ]
        body_lines += [
            f"const {it} phew_row = phew_g * blockDim.y + threadIdx.y;",
            "const bool phew_active = phew_row < phew_rows;",
            f"const {it} phew_lrow = phew_lrow0 + ({it})phew_buf * {buf}{u};",
        ]
        body_lines += self._row_reduce_lines(rplan, reduce_ext, r_names, r_dts, r_classes, out_shape, op,
                                             "", it, u, staged=staged, header=False)
        body_lines += [
            "if (threadIdx.x == 0) {",
            ("  phew_acc = __fdiv_rn(phew_acc, (float)phew_red);" if op == "mean" else ""),
            f"  phew_rowv_s[threadIdx.y] = phew_st_{_suffix(red_dt)}(phew_acc);",
            "}",
            "__syncthreads();",
            "if (phew_active) {",
        ]
        inner: list[str] = [
            f"const {CTYPE[red_dt]} phew_rowv[1] = {{phew_rowv_s[threadIdx.y]}};",
            f"const {it} phew_base = phew_row * phew_red;",
        ]
        scalar = self._scalar_body(mplan, map_ext, m_names, ["out0"], m_dts, [out_dt], m_classes,
                                   out_shape, it, u, staged=staged)
        if vec_ok:
            ptrs = " | ".join(f"reinterpret_cast<phew_uptr>({nm})" for nm in names + ["out0"]
                              if nm not in staged)
            vbody = self._vector_body(mplan, map_ext, m_names, ["out0"], m_dts, [out_dt], m_classes,
                                      out_shape, V, it, u, half_t, staged=staged)
            inner.append(f"if ((({ptrs}) & 15u) == 0u) {{")
            inner.append(f"  for ({it} phew_v = threadIdx.x; phew_v < phew_red / {V}{u}; phew_v += blockDim.x) {{")
            inner.append(f"    const {it} phew_off = phew_v * {V}{u};")
            inner.append(f"    const {it} elem = phew_base + phew_off;")
            inner += ["    " + b for b in vbody]
            inner.append("  }")
            inner.append("} else {")
        else:
            inner.append("{")
        inner.append(f"  for ({it} phew_c = threadIdx.x; phew_c < phew_red; phew_c += blockDim.x) {{")
        inner.append(f"    const {it} phew_off = phew_c;")
        inner.append(f"    const {it} elem = phew_base + phew_c;")
        inner += ["    " + b for b in scalar]
        inner.append("  }")
        inner.append("}")
        body_lines += ["  " + b for b in inner]
        body_lines += [
            "}",
            "__syncthreads();  // the buffer is refilled two groups from now",
        ]
        L += ["  " + b for b in body_lines]
        L.append("}")
        if staged:
            L.append("phew_cp_wait0();")
        source = "\n".join(f"    {line}" if line else "" for line in L)
        return source, names, ["out0"]

    # -- per-element form -----------------------------------------------------

    def _index(self, cls, ext, name, node, out_shape, it, u, elem="elem") -> str:
        if cls == "full":
            return elem
        if cls == "scalar":
            return "0"
        if cls == "suffix":
            return f"{elem} % {ext}{u}"
        if cls == "prefix":
            return f"{elem} / {ext}{u}"
        return general_index(elem, out_shape, tuple(int(s) for s in node.shape), it)

    def _scalar_body(self, plan, ext_in, inp_names, out_names, in_dts, out_dts, classes,
                     out_shape, it, u, staged: dict | None = None) -> list[str]:
        """Per-element statements for `elem`; a full-size input named in
        `staged` is read from its shared-memory row copy at
        ``phew_lrow + phew_off`` instead."""
        staged = staged or {}
        lines = []
        env = {}
        for node, nm, dt, (cls, ext) in zip(ext_in, inp_names, in_dts, classes):
            v = plan.var(node)
            if nm in staged and cls == "full":
                lines.append(f"const {VALUE_CTYPE[dt]} {v} = phew_ld({staged[nm]}[phew_lrow + phew_off]);")
                env[node.id] = (v, dt)
                continue
            idx = self._index(cls, ext, nm, node, out_shape, it, u)
            lines.append(f"const {VALUE_CTYPE[dt]} {v} = phew_ld({nm}[{idx}]);")
            env[node.id] = (v, dt)
        lines += plan.scalar_lines(env)
        for node, nm, dt in zip(plan.outputs, out_names, out_dts):
            v, vdt = env[node.id]
            lines.append(f"{nm}[elem] = phew_st_{_suffix(dt)}({_convert(v, vdt, dt)});")
        return lines

    # -- vector form ----------------------------------------------------------

    def _vector_body(self, plan, ext_in, inp_names, out_names, in_dts, out_dts, classes,
                     out_shape, V, it, u, half_t, staged: dict | None = None) -> list[str]:
        staged = staged or {}
        lines = []
        packed = half_t is not None and V == 8
        # Loads.
        for k, (node, nm, dt, (cls, ext)) in enumerate(zip(ext_in, inp_names, in_dts, classes)):
            ct = CTYPE[dt]
            if cls == "full" and nm in staged:
                lines.append(
                    f"const phew_vec<{ct}, {V}> ld{k} = phew_ldv_s<{ct}, {V}>({staged[nm]} + phew_lrow + phew_off);")
            elif cls == "full":
                lines.append(f"const phew_vec<{ct}, {V}> ld{k} = phew_ldv<{ct}, {V}>({nm} + elem);")
            elif cls == "suffix":
                lines.append(
                    f"const phew_vec<{ct}, {V}> ld{k} = phew_ldv<{ct}, {V}>({nm} + elem % {ext}{u});"
                )
            elif cls in ("scalar", "prefix"):
                idx = "0" if cls == "scalar" else f"elem / {ext}{u}"
                lines.append(f"const {ct} ld{k} = {nm}[{idx}];")
            else:
                lines.append(f"phew_vec<{ct}, {V}> ld{k};")
                lines.append("#pragma unroll")
                lines.append(f"for (int l = 0; l < {V}; ++l) {{")
                gi = general_index(f"(elem + l)", out_shape, tuple(int(s) for s in node.shape), it)
                lines.append(f"  ld{k}.v[l] = {nm}[{gi}];")
                lines.append("}")
        for k, (nm, dt) in enumerate(zip(out_names, out_dts)):
            lines.append(f"phew_vec<{CTYPE[dt]}, {V}> st{k};")
        if packed:
            P = V // 2
            lines.append("#pragma unroll")
            lines.append(f"for (int p = 0; p < {P}; ++p) {{")
            env = {}
            for k, (node, (cls, _)) in enumerate(zip(ext_in, classes)):
                v = plan.var(node)
                if cls in ("scalar", "prefix"):
                    lines.append(f"  const phew_u32 {v} = phew_splat2(ld{k});")
                else:
                    lines.append(f"  const phew_u32 {v} = phew_pair(ld{k}, p);")
                env[node.id] = v
            lines += ["  " + s for s in plan.packed_lines(env, half_t)]
            for k, node in enumerate(plan.outputs):
                lines.append(f"  phew_set_pair(st{k}, p, {env[node.id]});")
            lines.append("}")
        else:
            lines.append("#pragma unroll")
            lines.append(f"for (int l = 0; l < {V}; ++l) {{")
            env = {}
            for k, (node, dt, (cls, _)) in enumerate(zip(ext_in, in_dts, classes)):
                v = plan.var(node)
                src = f"ld{k}" if cls in ("scalar", "prefix") else f"ld{k}.v[l]"
                lines.append(f"  const {VALUE_CTYPE[dt]} {v} = phew_ld({src});")
                env[node.id] = (v, dt)
            lines += ["  " + s for s in plan.scalar_lines(env)]
            for k, (node, dt) in enumerate(zip(plan.outputs, out_dts)):
                v, vdt = env[node.id]
                lines.append(f"  st{k}.v[l] = phew_st_{_suffix(dt)}({_convert(v, vdt, dt)});")
            lines.append("}")
        for k, (nm, dt) in enumerate(zip(out_names, out_dts)):
            lines.append(f"phew_stv<{CTYPE[dt]}, {V}>({nm} + elem, st{k});")
        return lines


def _suffix(dt: str) -> str:
    return {"float32": "f32", "float16": "f16", "bfloat16": "bf16"}.get(dt, "raw")


def _convert(v: str, src: str, dst: str) -> str:
    if src == dst:
        return v
    return cast_expr(v, src, dst)


class _Plan:
    """Resolved chain: variable names, node order and dtype bookkeeping."""

    def __init__(self, nodes, ext_in, ext_out, precise16: bool = False, prefix: str = "v") -> None:
        self.precise16 = precise16
        self.prefix = prefix
        self.nodes = list(nodes)
        self.ext_in = list(ext_in)
        self.outputs = list(ext_out)
        self._names: dict[int, str] = {}
        self._ctr = 0
        for x in self.ext_in:
            self.var(x)
        self.compute_nodes = []
        self.constants = []
        for node in self.nodes:
            kind = node_kind(node)
            dt = dtype_name(node.dtype)
            if dt not in CTYPE:
                raise ValueError(f"cuda_codegen: unsupported dtype {dt!r}")
            if kind == "Constant":
                _const_literal(getattr(node, "value", None), dt)  # validates
                self.constants.append(node)
            elif kind == "Cast":
                tdt = dtype_name(getattr(node, "target_dtype", node.dtype))
                if tdt not in CTYPE:
                    raise ValueError(f"cuda_codegen: unsupported dtype {tdt!r}")
                self.compute_nodes.append(node)
            elif kind == "Elementwise":
                op = canonical_op(node.op)
                if op not in SUPPORTED_OPS and op not in ALIASES.values():
                    raise ValueError(f"cuda_codegen: unhandled op {node.op!r}")
                self.compute_nodes.append(node)
            else:
                raise ValueError(f"cuda_codegen: cannot fuse node kind {kind!r}")
            self.var(node)
        known = {x.id for x in self.ext_in} | {n.id for n in self.nodes}
        for node in self.nodes:
            for i in getattr(node, "inputs", []):
                if i not in known:
                    raise ValueError(f"cuda_codegen: input {i} of node {node.id} is not available")
        # Validate ops and arities by generating the scalar form once.
        env = {x.id: (self.var(x), dtype_name(x.dtype)) for x in self.ext_in}
        self.scalar_lines(env)
        for o in self.outputs:
            if o.id not in env:
                raise ValueError(f"cuda_codegen: output {o.id} is not computed by the chain")

    def var(self, node) -> str:
        if node.id not in self._names:
            self._ctr += 1
            self._names[node.id] = f"{self.prefix}{self._ctr}"
        return self._names[node.id]

    def pure_half_type(self, in_dts, out_dts) -> str | None:
        dts = set(in_dts) | set(out_dts)
        for node in self.nodes:
            dts.add(dtype_name(node.dtype))
            if node_kind(node) == "Cast":
                dts.add(dtype_name(getattr(node, "target_dtype", node.dtype)))
        if len(dts) == 1 and next(iter(dts)) in HALF_TYPES:
            return next(iter(dts))
        return None

    def constant_lines(self, packed_type: str | None) -> list[str]:
        lines = []
        for node in self.constants:
            dt = dtype_name(node.dtype)
            v = self.var(node)
            lit = _const_literal(node.value, dt)
            lines.append(f"const {VALUE_CTYPE[dt]} {v} = {lit};")
            if packed_type is not None and dt == packed_type:
                bits = half_bits(float(node.value), dt)
                lines.append(f"const phew_u32 {v}_x2 = 0x{bits:04x}{bits:04x}u;")
        return lines

    def scalar_lines(self, env: dict) -> list[str]:
        lines = []
        for node in self.constants:
            env[node.id] = (self.var(node), dtype_name(node.dtype))
        for node in self.compute_nodes:
            kind = node_kind(node)
            dt = dtype_name(node.dtype)
            v = self.var(node)
            args = [env[i] for i in node.inputs]
            if kind == "Cast":
                tdt = dtype_name(getattr(node, "target_dtype", node.dtype))
                expr = cast_expr(args[0][0], args[0][1], tdt)
                dt = tdt
            else:
                op = canonical_op(node.op)
                _check_arity(op, len(args))
                expr = scalar_expr(op, [a[0] for a in args], [a[1] for a in args], dt,
                                   precise16=self.precise16)
            lines.append(f"const {VALUE_CTYPE[dt]} {v} = {expr};")
            env[node.id] = (v, dt)
        return lines

    def packed_lines(self, env: dict, ht: str) -> list[str]:
        """Statements on packed pairs (phew_u32 holding two `ht` values)."""
        pfx = "phew_h2" if ht == "float16" else "phew_b2"
        lines = []
        for node in self.constants:
            env[node.id] = f"{self.var(node)}_x2"
        for node in self.compute_nodes:
            v = self.var(node)
            ins = [env[i] for i in node.inputs]
            if node_kind(node) == "Cast":
                lines.append(f"const phew_u32 {v} = {ins[0]};")
                env[node.id] = v
                continue
            op = canonical_op(node.op)
            _check_arity(op, len(ins))
            if op in _PACKED_NATIVE:
                nat = _PACKED_NATIVE[op]
                if nat == "sq":
                    lines.append(f"const phew_u32 {v} = {pfx}_mul({ins[0]}, {ins[0]});")
                elif nat in ("neg", "abs"):
                    lines.append(f"const phew_u32 {v} = {pfx}_{nat}({ins[0]});")
                else:
                    lines.append(f"const phew_u32 {v} = {pfx}_{nat}({ins[0]}, {ins[1]});")
            else:
                # Unpack, apply the scalar form to each half, repack.
                lo = [f"{pfx}_lo({a})" for a in ins]
                hi = [f"{pfx}_hi({a})" for a in ins]
                dts = [ht] * len(ins)
                # The pack conversion rounds each half to ht.
                e_lo = scalar_expr(op, lo, dts, ht, round_result=False, precise16=self.precise16)
                e_hi = scalar_expr(op, hi, dts, ht, round_result=False, precise16=self.precise16)
                lines.append(f"const phew_u32 {v} = {pfx}_pack({e_lo}, {e_hi});")
            env[node.id] = v
        return lines


_ARITY = {"where": 3}


def _check_arity(op: str, n: int) -> None:
    if op == "where":
        if n != 3:
            raise ValueError("cuda_codegen: where needs 3 inputs")
    elif op in _BINARY_F or op in _COMPARE or op in _LOGICAL or op in _BITWISE:
        if n != 2:
            raise ValueError(f"cuda_codegen: {op} needs 2 inputs, got {n}")
    elif n != 1:
        raise ValueError(f"cuda_codegen: {op} needs 1 input, got {n}")
