#!/usr/bin/env python3
"""Kernel IR -> B200 launch plan.

Usage:
    python compile.py path/to/<kernel>.ir.json > plan.json

Drop-in for the reference CLI (reference ``compile.py:70-106``): same
argument, same ``meta.json`` lookup beside the IR (``find_meta``), same
single-``KernelOp`` rule (``find_kernel``), same exit codes (2 usage, 1 any
``CompileError`` or invalid input, 0 success), same ``compile.py: <msg>``
stderr format with an empty stdout on failure, ASCII-only and deterministic
output.  What it prints is the launch plan of the sm_100a kernel family the
IR is (family, library symbol, tensor roles, view and scalars), which
``ptxc.launch.run`` executes; the reference printed PTX for a task runner that
no longer exists.
"""

from __future__ import annotations

import json
import os
import sys

sys.dont_write_bytecode = True
sys.path.insert(0, os.path.join(os.path.dirname(os.path.abspath(__file__)),
                                "emmy-ptx-compiler-submission_b200"))

from ptxc import CompileError, Lowerer  # noqa: E402


def find_kernel(graph):
    kernels = [node.op for node in graph.nodes.values()
               if type(node.op).__name__ == "KernelOp"]
    if not kernels:
        raise CompileError("graph contains no KernelOp")
    if len(kernels) > 1:
        raise CompileError(
            f"graph contains {len(kernels)} KernelOp nodes; expected exactly one")
    return kernels[0]


def find_meta(ir_path: str, entry: str):
    """The launch descriptor next to the IR, for this kernel (reference ``compile.py:35-67``)."""
    path = os.path.join(os.path.dirname(os.path.abspath(ir_path)), "meta.json")
    if not os.path.exists(path):
        return None
    try:
        with open(path) as fh:
            meta = json.load(fh)
    except (OSError, ValueError, RecursionError) as exc:
        raise CompileError(f"cannot read {path}: {exc}") from exc
    if not isinstance(meta, dict):
        raise CompileError(f"{path}: meta.json must be a JSON object")
    kernels = meta.get("kernels") or []
    if not isinstance(kernels, list):
        raise CompileError(f"{path}: meta.json kernels must be a list")
    if not kernels:
        raise CompileError(f"{path}: meta.json contains no kernels")
    for kernel in kernels:
        if not isinstance(kernel, dict):
            raise CompileError(f"{path}: each meta.json kernel must be an object")
    for kernel in kernels:
        if kernel.get("entry") == entry:
            return kernel
    names = ", ".join(str(k.get("entry")) for k in kernels)
    raise CompileError(f"meta.json has no kernel named {entry!r}; entries: {names}")


def load_ir(ir_path: str):
    """Parse the IR document with the clean-room loader; errors become CompileError."""
    from emmy_ir import Graph

    try:
        with open(ir_path) as fh:
            return Graph.from_dict(json.load(fh))
    except OSError as exc:
        raise CompileError(f"cannot read {ir_path}: {exc}") from exc
    except (json.JSONDecodeError, ValueError, TypeError, KeyError, AttributeError,
            NameError, SyntaxError, RecursionError) as exc:
        raise CompileError(f"invalid IR {ir_path}: {exc}") from exc


def compile_file(ir_path: str) -> str:
    graph = load_ir(ir_path)
    kernel_op = find_kernel(graph)
    meta = find_meta(ir_path, kernel_op.name)
    if meta is None:
        raise CompileError(
            f"meta.json not found next to {ir_path}; the launch descriptor is required")
    text = Lowerer(kernel_op, meta).compile()
    if not text.isascii():
        raise CompileError("launch plan must be ASCII")
    return text


def main(argv: list[str]) -> int:
    if len(argv) != 2:
        print("usage: python compile.py <kernel.ir.json>", file=sys.stderr)
        return 2
    try:
        text = compile_file(argv[1])
        sys.stdout.write(text)
    except CompileError as exc:
        print(f"compile.py: {exc}", file=sys.stderr)
        return 1
    except (TypeError, AttributeError, KeyError, IndexError, ValueError, OverflowError,
            RecursionError) as exc:
        print(f"compile.py: invalid input: {exc}", file=sys.stderr)
        return 1
    return 0


if __name__ == "__main__":
    sys.exit(main(sys.argv))
