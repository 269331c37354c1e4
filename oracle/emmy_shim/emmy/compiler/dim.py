"""``emmy.compiler.dim`` (reference call sites: ``ptxc/stmts.py:1095``, ``ptxc/expr.py:367,434,508``)."""
from emmy_ir.nodes import Dim  # noqa: F401
