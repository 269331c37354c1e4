"""Kernel IR vocabulary: frozen dataclasses for every statement and expression class.

The reference compiler consumes these objects through attribute names and
``type(obj).__name__`` only (``ptxc/common.py:27-28`` ``stmt_name``,
``ptxc/common.py:119-120`` ``_op_name``), so the field names and their order
below follow the keyword spelling used in the serialized IR (the ``repr``
strings inside ``KernelOp.op_fields.body``).  Every class is hashable and
supports ``dataclasses.replace``.  Expressions expose ``free_vars()``, which the
reference calls on index expressions (``ptxc/common.py:428``,
``ptxc/stmts.py:399``).
"""

from __future__ import annotations

from dataclasses import dataclass, field
from typing import Any


# ---------------------------------------------------------------------------
# leaf helpers


@dataclass(frozen=True)
class Dim:
    """A static extent.  ``Dim(128).value == 128`` (read as ``axis.extent.value``)."""
    value: int

    def __int__(self) -> int:
        return int(self.value)


@dataclass(frozen=True)
class NpDType:
    """Stand-in for the ``dtype('float32')`` call inside a serialized ``DataType``."""
    name: str

    def __str__(self) -> str:
        return self.name


@dataclass(frozen=True)
class DataType:
    name: str
    np: Any = None
    nbytes: int = 0

    def __str__(self) -> str:
        return self.name


@dataclass(frozen=True)
class ElementwiseImpl:
    """An elementwise op by name (``add``, ``exp``, ``reciprocal`` ...)."""
    name: str

    def __str__(self) -> str:
        return self.name


# ---------------------------------------------------------------------------
# expressions


class Expr:
    """Base class of index / predicate expressions."""

    def free_vars(self) -> frozenset:
        return frozenset()


@dataclass(frozen=True)
class Var(Expr):
    name: str

    def free_vars(self) -> frozenset:
        return frozenset((self.name,))


@dataclass(frozen=True)
class Literal(Expr):
    value: Any
    dtype: str = "int"

    def free_vars(self) -> frozenset:
        return frozenset()


@dataclass(frozen=True)
class BinaryExpr(Expr):
    op: str
    left: Any
    right: Any

    def free_vars(self) -> frozenset:
        out = frozenset()
        for side in (self.left, self.right):
            if isinstance(side, Expr):
                out |= side.free_vars()
        return out


@dataclass(frozen=True)
class TernaryExpr(Expr):
    cond: Any
    if_true: Any
    if_false: Any

    def free_vars(self) -> frozenset:
        out = frozenset()
        for side in (self.cond, self.if_true, self.if_false):
            if isinstance(side, Expr):
                out |= side.free_vars()
        return out


@dataclass(frozen=True)
class CastExpr(Expr):
    expr: Any
    dtype: Any = None

    def free_vars(self) -> frozenset:
        return self.expr.free_vars() if isinstance(self.expr, Expr) else frozenset()


@dataclass(frozen=True)
class Builtin(Expr):
    name: str

    def free_vars(self) -> frozenset:
        return frozenset()


@dataclass(frozen=True)
class FlatIndex(Expr):
    buffer: Any
    index: Any = ()

    def free_vars(self) -> frozenset:
        out = frozenset()
        for e in self.index or ():
            if isinstance(e, Expr):
                out |= e.free_vars()
        return out


# ---------------------------------------------------------------------------
# axes and statements


@dataclass(frozen=True)
class Window:
    parent: Any = None
    base: Any = None
    bound: Any = None
    partition: bool = False


@dataclass(frozen=True)
class Axis:
    name: str
    extent: Any
    window: Any = None


@dataclass(frozen=True)
class Tile:
    axes: tuple
    body: tuple
    block_threads: int = 0
    aux_threads: int = 0
    raster_axes: Any = None
    raster_group: Any = None
    raster_orient: str = "m"


@dataclass(frozen=True)
class Loop:
    axis: Axis
    body: tuple
    unroll: bool = False
    seed: bool = True


@dataclass(frozen=True)
class StridedLoop:
    axis: Axis
    start: Any
    step: Any
    body: tuple
    unroll: bool = False
    end: Any = None
    seed: bool = True


@dataclass(frozen=True)
class Load:
    names: tuple
    input: str
    index: tuple
    dtype: Any = None


@dataclass(frozen=True)
class Write:
    output: str
    index: tuple
    values: tuple
    value_dtype: Any = None
    atomic: bool = False
    swizzle: str = "NONE"


@dataclass(frozen=True)
class Assign:
    name: str
    op: Any
    args: tuple
    dtype: Any = None


@dataclass(frozen=True)
class Accum:
    name: str
    value: str
    op: Any
    dtype: Any = None
    axes: tuple = ()
    base: Any = None


@dataclass(frozen=True)
class Let:
    name: str
    value: Any
    dtype: Any = None


@dataclass(frozen=True)
class Init:
    name: str
    identity: Any
    dtype: Any = None


@dataclass(frozen=True)
class Smem:
    name: str
    extents: tuple
    dtype: str = "float"
    align: int = 0


@dataclass(frozen=True)
class Cond:
    cond: Any
    body: tuple = ()
    else_body: tuple = ()


@dataclass(frozen=True)
class Sync:
    barrier_id: int = 0
    count: Any = None
    warp: bool = False


@dataclass(frozen=True)
class WarpShuffle:
    state: tuple
    state_b: tuple
    combine_states: tuple
    length: int = 32
    dtype: Any = None


@dataclass(frozen=True)
class TreeHalve:
    bufs: tuple
    state: tuple
    state_b: tuple
    combine_states: tuple
    length: int
    tid_var: str = "warp"
    dtype: Any = None
    barrier_id: int = 0
    barrier_count: Any = None
    inner: Any = None


@dataclass(frozen=True)
class CpAsyncCopy:
    smem: str
    smem_index: tuple
    src: str
    src_index: tuple
    nbytes: int = 16
    swizzle: str = "NONE"
    lane_index: Any = None
    lane_rows: int = 0


@dataclass(frozen=True)
class CpAsyncCommit:
    pass


@dataclass(frozen=True)
class CpAsyncWait:
    group: int = 0


@dataclass(frozen=True)
class ZeroPrologue:
    dst: str
    words: Any = None


@dataclass(frozen=True)
class KernelOp:
    """The one kernel of a graph: ``name`` is the PTX entry, ``body`` its statements."""
    name: str
    body: tuple
    zero_delegated: tuple = ()
    serial: tuple = ()


@dataclass(frozen=True)
class InputOp:
    pass


@dataclass(frozen=True)
class ConstantOp:
    name: str = ""
    value: Any = None
    context_value: Any = None
    load_ops: tuple = ()
    source_path: Any = None
    source_parts: tuple = ()
    source_shape: Any = None
    source_dtype: Any = None
    source_graph: Any = None


# Every class name the serialized statement strings may construct.  The parser
# accepts these and nothing else (plus the ``dtype`` helper).
IR_CLASSES = {
    cls.__name__: cls
    for cls in (
        Dim, DataType, ElementwiseImpl, Var, Literal, BinaryExpr, TernaryExpr,
        CastExpr, Builtin, FlatIndex, Window, Axis, Tile, Loop, StridedLoop,
        Load, Write, Assign, Accum, Let, Init, Smem, Cond, Sync, WarpShuffle,
        TreeHalve, CpAsyncCopy, CpAsyncCommit, CpAsyncWait, ZeroPrologue,
    )
}

STATEMENT_CLASSES = frozenset({
    "Tile", "Loop", "StridedLoop", "Load", "Write", "Assign", "Accum", "Let",
    "Init", "Smem", "Cond", "Sync", "WarpShuffle", "TreeHalve", "CpAsyncCopy",
    "CpAsyncCommit", "CpAsyncWait", "ZeroPrologue",
})


def dtype_name(dt) -> str:
    """Normalise a dtype field (``DataType``, C spelling, or ``None``) to an emmy name.

    Follows ``ptxc/ops.py:40-45`` (``norm_dtype``): ``None`` reads as f32 and the
    C spellings used by ``Smem.dtype`` map onto emmy names.
    """
    if dt is None:
        return "f32"
    name = str(getattr(dt, "name", dt))
    return C_DTYPES.get(name, name)


# C spellings that appear in Smem.dtype (``ptxc/ops.py:27-37``).
C_DTYPES = {
    "float": "f32",
    "double": "f64",
    "half": "f16",
    "__half": "f16",
    "int": "i32",
    "unsigned": "u32",
    "long": "i64",
    "short": "i16",
    "char": "i8",
}


def iter_stmts(stmts):
    """Depth-first walk over statements, including Cond/Loop bodies (not combine_states)."""
    for st in stmts or ():
        yield st
        for attr in ("body", "else_body"):
            child = getattr(st, attr, None)
            if isinstance(child, (tuple, list)) and child:
                yield from iter_stmts(child)
