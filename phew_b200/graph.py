"""Plain records of phew μGraph nodes.

The backend reads phew's IR by duck typing (class name, ``id``, ``shape``,
``dtype``, ``inputs`` and the op fields of ``phew.ir.ops``, ``ir/ops.py``).
``NodeSpec`` carries the same fields without importing phew, so fused chains
and graphs can be built, stored as JSON fixtures and replayed where phew is
not installed.  ``from_phew`` converts a live ``phew.ir.Graph``.
"""

from __future__ import annotations

import itertools
import json
from dataclasses import dataclass, field
from typing import Any

_ids = itertools.count(1_000_000)

# Fields of phew.ir.ops node classes that the backend reads.
OP_FIELDS = (
    "op", "axes", "keepdims", "value", "target_dtype", "name", "eps", "scale", "mask",
    "transpose_a", "transpose_b", "new_shape", "input_shape", "output_idx", "source",
    "header", "input_names", "output_names", "output_shapes", "output_dtypes",
    "input_shapes", "threadgroup", "grid", "template_params",
)


@dataclass
class NodeSpec:
    """One μGraph node: ``kind`` is the phew.ir.ops class name."""

    kind: str
    shape: tuple = ()
    dtype: str = "float32"
    inputs: list = field(default_factory=list)
    attrs: dict = field(default_factory=dict)
    id: int = field(default_factory=lambda: next(_ids))
    op: str | None = None
    value: Any = None
    target_dtype: str | None = None
    name: str | None = None

    def __getattr__(self, item):  # other op fields live in attrs
        attrs = self.__dict__.get("attrs", {})
        if item in attrs:
            return attrs[item]
        raise AttributeError(item)

    @property
    def numel(self) -> int:
        n = 1
        for s in self.shape:
            n *= int(s)
        return n

    def to_json(self) -> dict:
        d = {"kind": self.kind, "id": self.id, "shape": list(self.shape), "dtype": self.dtype,
             "inputs": list(self.inputs)}
        for k in ("op", "value", "target_dtype", "name"):
            v = getattr(self, k)
            if v is not None:
                d[k] = v
        if self.attrs:
            d["attrs"] = _jsonable(self.attrs)
        return d

    @classmethod
    def from_json(cls, d: dict) -> "NodeSpec":
        return cls(
            kind=d["kind"], shape=tuple(d.get("shape", ())), dtype=d.get("dtype", "float32"),
            inputs=list(d.get("inputs", [])), attrs=dict(d.get("attrs", {})), id=int(d["id"]),
            op=d.get("op"), value=d.get("value"), target_dtype=d.get("target_dtype"),
            name=d.get("name"),
        )


def _jsonable(v):
    if isinstance(v, dict):
        return {str(k): _jsonable(x) for k, x in v.items()}
    if isinstance(v, (list, tuple)):
        return [_jsonable(x) for x in v]
    if hasattr(v, "value") and isinstance(getattr(v, "value"), str):
        return v.value
    if isinstance(v, (str, int, float, bool)) or v is None:
        return v
    return repr(v)


class GraphSpec:
    """Ordered node records with phew Graph's query methods."""

    def __init__(self, nodes: list[NodeSpec] | None = None, outputs: list[int] | None = None):
        self._nodes: dict[int, NodeSpec] = {}
        for n in nodes or []:
            self._nodes[n.id] = n
        self.outputs: list[int] = list(outputs or [])

    def add(self, node: NodeSpec) -> NodeSpec:
        self._nodes[node.id] = node
        return node

    def __getitem__(self, nid: int) -> NodeSpec:
        return self._nodes[nid]

    def __contains__(self, nid: int) -> bool:
        return nid in self._nodes

    def __len__(self) -> int:
        return len(self._nodes)

    def nodes(self) -> list[NodeSpec]:
        return list(self._nodes.values())

    def inputs(self) -> list[NodeSpec]:
        return [n for n in self._nodes.values() if n.kind == "Input"]

    def topo_order(self) -> list[NodeSpec]:
        seen: set[int] = set()
        out: list[NodeSpec] = []

        def visit(nid: int) -> None:
            if nid in seen or nid not in self._nodes:
                return
            seen.add(nid)
            for i in self._nodes[nid].inputs:
                visit(i)
            out.append(self._nodes[nid])

        for nid in self.outputs or list(self._nodes):
            visit(nid)
        return out

    def successors(self, nid: int) -> list[NodeSpec]:
        return [n for n in self._nodes.values() if nid in n.inputs]

    def to_json(self) -> dict:
        return {"nodes": [n.to_json() for n in self._nodes.values()], "outputs": self.outputs}

    @classmethod
    def from_json(cls, d: dict | str) -> "GraphSpec":
        if isinstance(d, str):
            d = json.loads(d)
        return cls([NodeSpec.from_json(x) for x in d["nodes"]], d["outputs"])


def from_phew(graph) -> GraphSpec:
    """Record a live phew.ir.Graph (duck-typed; phew need not be importable)."""
    specs = []
    for node in graph.nodes():
        kind = type(node).__name__
        attrs = {}
        for f in OP_FIELDS:
            if f in ("op", "value", "target_dtype", "name"):
                continue
            if hasattr(node, f):
                attrs[f] = _jsonable(getattr(node, f))
        if getattr(node, "attrs", None):
            attrs["node_attrs"] = _jsonable(node.attrs)
        dt = getattr(node.dtype, "value", node.dtype)
        spec = NodeSpec(kind=kind, shape=tuple(node.shape), dtype=str(dt), inputs=list(node.inputs),
                        attrs=attrs, id=node.id)
        if kind == "Elementwise" or kind == "Reduce":
            spec.op = node.op
        if kind == "Constant":
            spec.value = node.value
        if kind == "Cast":
            spec.target_dtype = getattr(node.target_dtype, "value", str(node.target_dtype))
        if kind == "Input":
            spec.name = node.name
        specs.append(spec)
    return GraphSpec(specs, list(graph.outputs))


# -- small builders used by workloads and tests ------------------------------


def inp(shape, dtype, name) -> NodeSpec:
    return NodeSpec("Input", tuple(shape), dtype, name=name)


def const(value, dtype) -> NodeSpec:
    return NodeSpec("Constant", (), dtype, value=value)


def ew(op, *ins, shape=None, dtype=None) -> NodeSpec:
    shape = tuple(shape if shape is not None else _bshape(*[i.shape for i in ins]))
    dtype = dtype or ins[0].dtype
    return NodeSpec("Elementwise", shape, dtype, inputs=[i.id for i in ins], op=op)


def cast(x, dtype) -> NodeSpec:
    return NodeSpec("Cast", tuple(x.shape), dtype, inputs=[x.id], target_dtype=dtype)


def _bshape(*shapes):
    nd = max(len(s) for s in shapes)
    out = []
    for i in range(nd):
        d = 1
        for s in shapes:
            p = (1,) * (nd - len(s)) + tuple(s)
            if p[i] != 1:
                d = p[i]
        out.append(d)
    return tuple(out)
