"""``Graph.from_dict``: the IR document loader the CLI calls.

Replaces the third-party ``emmy.compiler.graph.Graph`` that the reference
imports at ``compile.py:76``.  The document shape (``inputs``, ``outputs``,
``nodes`` of ``{op, op_fields, inputs, outputs}``) is the one every
``tests/variants/*/*.ir.json`` of the reference carries.  Exposes the surface
the reference reads: ``graph.nodes[name].op`` with ``type(op).__name__ ==
"KernelOp"`` and ``op.name`` / ``op.body`` (``compile.py:24-32``).

Malformed documents raise ``ValueError``/``TypeError``/``KeyError``, which
``compile.py`` maps to ``CompileError("invalid IR ...")`` exactly as the
reference does at ``compile.py:84-86``.
"""

from __future__ import annotations

from dataclasses import dataclass, field

from .nodes import ConstantOp, InputOp, KernelOp
from .parse import IRSyntaxError, parse_node


@dataclass(frozen=True)
class TensorSpec:
    name: str
    shape: tuple
    dtype: str


@dataclass
class Node:
    name: str
    op: object
    inputs: tuple
    outputs: tuple


@dataclass
class Graph:
    inputs: tuple = ()
    outputs: tuple = ()
    nodes: dict = field(default_factory=dict)

    @classmethod
    def from_dict(cls, doc) -> "Graph":
        if not isinstance(doc, dict):
            raise TypeError("IR document must be a JSON object")
        raw_nodes = doc["nodes"]
        if not isinstance(raw_nodes, dict):
            raise TypeError("IR nodes must be an object")
        nodes = {}
        for name, raw in raw_nodes.items():
            if not isinstance(raw, dict):
                raise TypeError(f"node {name!r} must be an object")
            kind = raw["op"]
            fields = raw.get("op_fields") or {}
            if not isinstance(fields, dict):
                raise TypeError(f"node {name!r} op_fields must be an object")
            if kind == "KernelOp":
                body = fields["body"]
                if not isinstance(body, list):
                    raise TypeError(f"KernelOp {name!r} body must be a list")
                op = KernelOp(
                    name=fields.get("name", name),
                    body=tuple(parse_node(s) for s in body),
                    zero_delegated=tuple(fields.get("zero_delegated") or ()),
                    serial=tuple(fields.get("serial") or ()),
                )
                if not isinstance(op.name, str):
                    raise TypeError(f"KernelOp {name!r} name must be a string")
            elif kind == "InputOp":
                op = InputOp()
            elif kind == "ConstantOp":
                known = {k: fields.get(k) for k in (
                    "name", "value", "context_value", "source_path", "source_shape",
                    "source_dtype", "source_graph")}
                known["load_ops"] = tuple(fields.get("load_ops") or ())
                known["source_parts"] = tuple(fields.get("source_parts") or ())
                op = ConstantOp(**known)
            else:
                raise ValueError(f"node {name!r} has unknown op {kind!r}")
            outs = []
            for o in raw.get("outputs") or ():
                if not isinstance(o, dict):
                    raise TypeError(f"node {name!r} outputs must be objects")
                outs.append(TensorSpec(o["name"], tuple(o.get("shape") or ()), o.get("dtype", "f32")))
            nodes[name] = Node(name, op, tuple(raw.get("inputs") or ()), tuple(outs))
        return cls(tuple(doc.get("inputs") or ()), tuple(doc.get("outputs") or ()), nodes)


__all__ = ["Graph", "Node", "TensorSpec", "IRSyntaxError"]
