"""Restricted parser for the ``repr`` strings that carry a KernelOp body.

The serialized IR stores each top-level statement as a Python ``repr`` string
of the emmy dataclass (for example the body strings of any
``tests/variants/*/*.ir.json`` in the reference).  The reference relies on the
third-party deserializer and maps its failures (``NameError``, ``SyntaxError``
and friends) to "invalid IR" (``compile.py:82-86``).  This module never calls
``eval``: it walks the ``ast`` of the string and only builds the whitelisted
classes of :mod:`emmy_ir.nodes`, from keyword or positional arguments, over
literals, tuples and lists.  Anything else raises :class:`IRSyntaxError`, a
``ValueError``, which the CLI reports as invalid IR.
"""

from __future__ import annotations

import ast
import dataclasses

from .nodes import IR_CLASSES, NpDType

MAX_DEPTH = 400


class IRSyntaxError(ValueError):
    pass


def parse_node(text: str):
    """Parse one statement string into IR objects."""
    if not isinstance(text, str):
        raise IRSyntaxError(f"statement must be a string, got {type(text).__name__}")
    try:
        tree = ast.parse(text, mode="eval")
    except SyntaxError as exc:
        raise IRSyntaxError(f"cannot parse statement: {exc.msg}") from exc
    except RecursionError as exc:
        raise IRSyntaxError("statement nests too deeply") from exc
    return _build(tree.body, 0)


def _build(node, depth: int):
    if depth > MAX_DEPTH:
        raise IRSyntaxError("statement nests too deeply")
    if isinstance(node, ast.Constant):
        if isinstance(node.value, (int, float, str, bool)) or node.value is None:
            return node.value
        raise IRSyntaxError(f"unsupported constant {node.value!r}")
    if isinstance(node, ast.UnaryOp) and isinstance(node.op, (ast.USub, ast.UAdd)):
        inner = _build(node.operand, depth + 1)
        if isinstance(inner, bool) or not isinstance(inner, (int, float)):
            raise IRSyntaxError("unary sign on a non-number")
        return -inner if isinstance(node.op, ast.USub) else inner
    if isinstance(node, ast.Tuple):
        return tuple(_build(e, depth + 1) for e in node.elts)
    if isinstance(node, ast.List):
        return tuple(_build(e, depth + 1) for e in node.elts)
    if isinstance(node, ast.Name):
        if node.id in ("inf", "nan"):
            return float(node.id)
        raise IRSyntaxError(f"name {node.id!r} is not an IR class")
    if isinstance(node, ast.Call):
        if not isinstance(node.func, ast.Name):
            raise IRSyntaxError("only plain IR class constructors are allowed")
        name = node.func.id
        if name == "dtype":
            if len(node.args) != 1 or node.keywords:
                raise IRSyntaxError("dtype() takes one string")
            arg = _build(node.args[0], depth + 1)
            if not isinstance(arg, str):
                raise IRSyntaxError("dtype() takes one string")
            return NpDType(arg)
        if name == "float" and len(node.args) == 1 and not node.keywords:
            arg = _build(node.args[0], depth + 1)
            if arg in ("inf", "-inf", "nan"):
                return float(arg)
            raise IRSyntaxError("float() only spells inf or nan")
        cls = IR_CLASSES.get(name)
        if cls is None:
            raise IRSyntaxError(f"name {name!r} is not an IR class")
        args = [_build(a, depth + 1) for a in node.args]
        kwargs = {}
        for kw in node.keywords:
            if kw.arg is None:
                raise IRSyntaxError("** arguments are not allowed")
            kwargs[kw.arg] = _build(kw.value, depth + 1)
        fields = {f.name for f in dataclasses.fields(cls)}
        unknown = sorted(set(kwargs) - fields)
        if unknown:
            raise IRSyntaxError(f"{name} has no field(s) {', '.join(unknown)}")
        try:
            return cls(*args, **kwargs)
        except TypeError as exc:
            raise IRSyntaxError(f"bad arguments to {name}: {exc}") from exc
    raise IRSyntaxError(f"unsupported syntax {type(node).__name__}")
