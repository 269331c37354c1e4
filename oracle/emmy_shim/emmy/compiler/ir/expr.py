"""``emmy.compiler.ir.expr`` (reference call sites listed in ``ptxc/expr.py``, ``ptxc/stmts.py``,
``ptxc/memory.py``, ``ptxc/common.py``)."""
from emmy_ir.nodes import (  # noqa: F401
    BinaryExpr, Builtin, CastExpr, Expr, FlatIndex, Literal, TernaryExpr, Var,
)
