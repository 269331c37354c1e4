"""``emmy.compiler.graph`` (reference call site: ``compile.py:76``)."""
from emmy_ir.graph import Graph  # noqa: F401
