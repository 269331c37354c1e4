"""Clean-room IR loader: parses every reference fixture, round-trips, rejects non-IR."""

from __future__ import annotations

import json

import pytest

from conftest import load_variant, needs_reference, reference_variants
from emmy_ir import Graph, IRSyntaxError, parse_node
from emmy_ir.serialize import to_repr


@needs_reference
def test_every_fixture_parses_and_round_trips():
    paths = reference_variants()
    assert len(paths) == 46
    for p in paths:
        kop, meta, ir = load_variant(p)
        assert type(kop).__name__ == "KernelOp"
        assert kop.name == meta["kernels"][0]["entry"]
        doc = json.loads(ir.read_text())
        node = [n for n in doc["nodes"].values() if n["op"] == "KernelOp"][0]
        for text, st in zip(node["op_fields"]["body"], kop.body):
            assert to_repr(st) == text


@pytest.mark.parametrize("text", [
    "__import__('os').system('true')",
    "Tile(axes=(), body=(), block_threads=1, aux_threads=0, raster_axes=None, raster_group=None, raster_orient=open('x'))",
    "Var(name='a').__class__",
    "lambda: 0",
    "Var(**{'name': 'a'})",
    "Var(nome='a')",
    "[x for x in ()]",
])
def test_non_ir_syntax_is_rejected_without_eval(text):
    with pytest.raises(IRSyntaxError):
        parse_node(text)


def test_graph_errors_are_value_or_type_errors():
    with pytest.raises((ValueError, TypeError, KeyError)):
        Graph.from_dict({"nodes": {"k": {"op": "KernelOp", "op_fields": {"body": ["Nope()"], "name": "k"}}}})
    with pytest.raises((ValueError, TypeError, KeyError)):
        Graph.from_dict([])
    with pytest.raises((ValueError, TypeError, KeyError)):
        Graph.from_dict({"nodes": {"k": {"op": "MysteryOp"}}})


def test_expressions_are_hashable_and_report_free_vars():
    e = parse_node("BinaryExpr(op='+', left=Var(name='a0'), right=BinaryExpr(op='*', left=Var(name='b'), right=Literal(value=4, dtype='int')))")
    assert e.free_vars() == {"a0", "b"}
    assert hash(e) == hash(parse_node(to_repr(e)))
