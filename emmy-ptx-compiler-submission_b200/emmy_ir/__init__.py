"""Clean-room Kernel IR loader (``Graph.from_dict``) and IR vocabulary.

Stands in for the ``emmy-ml==0.3.11`` deserializer the reference imports
(``compile.py:76``); written from the serialized format alone and parsed with
an ``ast`` whitelist, never ``eval``.
"""

from .graph import Graph, Node, TensorSpec
from .nodes import *  # noqa: F401,F403
from .nodes import IR_CLASSES, STATEMENT_CLASSES, dtype_name, iter_stmts
from .parse import IRSyntaxError, parse_node

__all__ = ["Graph", "Node", "TensorSpec", "IRSyntaxError", "parse_node",
           "IR_CLASSES", "STATEMENT_CLASSES", "dtype_name", "iter_stmts"]
