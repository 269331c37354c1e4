"""B200 host layer for Emmy's Kernel IR: family matcher, launch plan, ctypes launcher.

Same public surface as the reference package (``ptxc/__init__.py``:
``Lowerer``, ``CompileError``).  ``Lowerer(kernel_op, meta).compile()`` returns
the launch plan text; ``ptxc.launch.run(plan, tensors)`` executes it on the GPU
through ``libemmyb200.so``.
"""

from .common import CompileError
from .lower import Lowerer

__all__ = ["Lowerer", "CompileError"]
