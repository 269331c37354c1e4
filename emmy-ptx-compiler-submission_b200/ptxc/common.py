"""Shared rules of the host layer: ``CompileError`` and the dtype table.

``CompileError`` is the one expected failure of the compile path, as in the
reference (``ptxc/common.py:115``); the CLI prints it as ``compile.py: <msg>``
and exits 1.  The dtype table keeps the reference's emmy dtype names and
widths (``ptxc/ops.py:11-25``) and its C spellings for shared buffers
(``ptxc/ops.py:27-37``).
"""

from __future__ import annotations


class CompileError(Exception):
    """The IR or its meta.json cannot be turned into a launch plan."""


# emmy dtype name -> byte width
DTYPES: dict[str, int] = {
    "f32": 4, "f16": 2, "f64": 8,
    "i8": 1, "u8": 1, "i16": 2, "u16": 2, "i32": 4, "u32": 4, "i64": 8, "u64": 8,
    "bool": 1,
}

C_DTYPES = {
    "float": "f32", "double": "f64", "half": "f16", "__half": "f16", "int": "i32",
    "unsigned": "u32", "long": "i64", "short": "i16", "char": "i8",
}


def norm_dtype(name) -> str:
    """``ptxc/ops.py:40-45``: ``None`` is f32, a ``DataType`` by its name, C spellings mapped."""
    if name is None:
        return "f32"
    name = str(getattr(name, "name", name))
    return C_DTYPES.get(name, name)


def check_dtype(dt: str, where: str) -> None:
    if dt not in DTYPES:
        raise CompileError(f"unsupported dtype {dt!r} in {where}")


def stmt_name(st) -> str:
    return type(st).__name__


def op_name(op) -> str:
    return getattr(op, "name", str(op))


def const_int(e):
    """Integer value of a Literal/Dim/int, else None (``ptxc/common.py:134-142``)."""
    if e is None:
        return None
    if isinstance(e, bool):
        return None
    if isinstance(e, int):
        return e
    value = getattr(e, "value", None)
    if isinstance(value, bool):
        return None
    if isinstance(value, int):
        return value
    if isinstance(value, float) and value.is_integer():
        return int(value)
    return None


def iter_stmts(stmts):
    for st in stmts or ():
        yield st
        for attr in ("body", "else_body"):
            child = getattr(st, attr, None)
            if isinstance(child, (tuple, list)) and child:
                yield from iter_stmts(child)
