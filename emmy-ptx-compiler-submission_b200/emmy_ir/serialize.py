"""Write IR objects back in the serialized format (``repr`` strings in JSON).

The inverse of :mod:`emmy_ir.parse`: dataclass instances print as
``ClassName(field=value, ...)`` in field order, ``Dim`` and
``ElementwiseImpl`` positionally, numpy dtypes as ``dtype('float32')`` --
the spelling of the body strings in the reference's
``tests/variants/*/*.ir.json``.  ``parse_node(to_repr(x)) == x`` for every
node.
"""

from __future__ import annotations

import dataclasses
import json
from pathlib import Path

from .nodes import Dim, ElementwiseImpl, KernelOp, NpDType


def to_repr(v) -> str:
    if isinstance(v, Dim):
        return f"Dim({int(v.value)})"
    if isinstance(v, ElementwiseImpl):
        return f"ElementwiseImpl({v.name!r})"
    if isinstance(v, NpDType):
        return f"dtype({v.name!r})"
    if dataclasses.is_dataclass(v) and not isinstance(v, type):
        parts = [f"{f.name}={to_repr(getattr(v, f.name))}" for f in dataclasses.fields(v)]
        return f"{type(v).__name__}(" + ", ".join(parts) + ")"
    if isinstance(v, tuple):
        inner = ", ".join(to_repr(x) for x in v)
        return "(" + inner + ("," if len(v) == 1 else "") + ")"
    if isinstance(v, list):
        return to_repr(tuple(v))
    if isinstance(v, (bool, int, float, str)) or v is None:
        return repr(v)
    raise TypeError(f"cannot serialise {type(v).__name__}")


def graph_dict(kernel: KernelOp, args: list, out_name: str) -> dict:
    """A one-kernel IR document: an InputOp/ConstantOp per argument, then the KernelOp.

    ``args`` are meta.json argument dicts (name, dtype, shape, data/seed/output).
    """
    nodes = {}
    inputs = []
    for a in args:
        if a.get("output"):
            continue
        if "data" in a:
            nodes[a["name"]] = {
                "op": "ConstantOp",
                "op_fields": {"name": a["name"], "value": a["data"][0] if len(a["data"]) == 1 else a["data"],
                              "context_value": None, "load_ops": [], "source_path": None,
                              "source_parts": [], "source_shape": None, "source_dtype": None,
                              "source_graph": None},
                "inputs": [],
                "outputs": [{"name": a["name"], "shape": list(a["shape"]), "dtype": a["dtype"]}],
            }
        else:
            inputs.append(a["name"])
            nodes[a["name"]] = {"op": "InputOp", "op_fields": {}, "inputs": [],
                                "outputs": [{"name": a["name"], "shape": list(a["shape"]),
                                             "dtype": a["dtype"]}]}
    out = [a for a in args if a["name"] == out_name][0]
    nodes[out_name] = {
        "op": "KernelOp",
        "op_fields": {"body": [to_repr(s) for s in kernel.body], "name": kernel.name,
                      "zero_delegated": list(kernel.zero_delegated), "serial": list(kernel.serial)},
        "inputs": [a["name"] for a in args if not a.get("output")],
        "outputs": [{"name": out_name, "shape": list(out["shape"]), "dtype": out["dtype"]}],
    }
    return {"inputs": sorted(inputs), "outputs": [out_name], "nodes": nodes}


def write_package(directory, kernel: KernelOp, meta_kernel: dict, package: dict | None = None) -> Path:
    """Write ``<entry>.ir.json`` and ``meta.json`` into ``directory``; returns the IR path."""
    d = Path(directory)
    d.mkdir(parents=True, exist_ok=True)
    outs = [a["name"] for a in meta_kernel["args"] if a.get("output")]
    doc = graph_dict(kernel, meta_kernel["args"], outs[0])
    ir_path = d / f"{kernel.name}.ir.json"
    ir_path.write_text(json.dumps(doc, indent=1))
    meta = dict(package or {})
    meta.setdefault("id", kernel.name)
    meta.setdefault("graph_inputs", [a["name"] for a in meta_kernel["args"]
                                     if not a.get("output") and "data" not in a])
    meta.setdefault("graph_outputs", outs)
    meta["kernels"] = [meta_kernel]
    (d / "meta.json").write_text(json.dumps(meta, indent=1))
    return ir_path


def write_chain(directory, pairs, package: dict | None = None) -> list:
    """A package of several kernels: one ``<entry>.ir.json`` each and one
    ``meta.json`` listing them in launch order; returns the IR paths."""
    d = Path(directory)
    d.mkdir(parents=True, exist_ok=True)
    paths = []
    for kernel, mk in pairs:
        outs = [a["name"] for a in mk["args"] if a.get("output")]
        doc = graph_dict(kernel, mk["args"], outs[0])
        path = d / f"{kernel.name}.ir.json"
        path.write_text(json.dumps(doc, indent=1))
        paths.append(path)
    meta = dict(package or {})
    meta.setdefault("id", pairs[-1][0].name)
    meta["kernels"] = [mk for _, mk in pairs]
    (d / "meta.json").write_text(json.dumps(meta, indent=1))
    return paths
