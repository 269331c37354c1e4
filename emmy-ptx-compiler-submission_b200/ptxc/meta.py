"""Strict ``meta.json`` kernel-entry validation.

Restates ``Lowerer._read_meta`` of the reference (``ptxc/lower.py:425-521``)
check for check and message for message, because the drop-in contract is
defined by those messages (the CLI tests look for ``shape``, ``dtype``,
``arg_order``, ``3 integers``, ``scalar``, ``arch``; reference
``tests/test_cli.py:69-115``).
"""

from __future__ import annotations

from .common import CompileError, check_dtype, norm_dtype


class MetaInfo:
    """The validated launch descriptor of one kernel."""

    def __init__(self, meta: dict):
        self.raw = meta
        self.shapes: dict[str, tuple] = {}
        self.dtypes: dict[str, str] = {}
        self.data: dict[str, list] = {}
        self.outputs: list[str] = []
        self.scalars: set[str] = set()
        self.grid: tuple = ()
        self.block: tuple = ()
        self.smem_bytes = 0
        self.arg_order: list[str] = []
        self.zero_outputs: list[str] = []


def read_meta(meta) -> MetaInfo:
    if not isinstance(meta, dict):
        raise CompileError("meta.json must be a JSON object")
    info = MetaInfo(meta)
    for key in ("grid", "block"):
        if key not in meta:
            raise CompileError(f"meta.json is missing {key}")
        raw = meta[key]
        if not isinstance(raw, (list, tuple)) or len(raw) != 3:
            raise CompileError(f"meta.json {key} must be a list of 3 integers")
        if any(isinstance(x, bool) or not isinstance(x, int) for x in raw):
            raise CompileError(f"meta.json {key} must contain integers: {raw!r}")
        if any(x <= 0 for x in raw):
            raise CompileError(f"meta.json {key} must contain positive integers: {raw!r}")
    info.grid = tuple(meta["grid"])
    info.block = tuple(meta["block"])
    raw_smem = meta.get("smem_bytes", 0)
    if raw_smem is None:
        raw_smem = 0
    if isinstance(raw_smem, bool) or not isinstance(raw_smem, int) or raw_smem < 0:
        raise CompileError("meta.json smem_bytes must be a non-negative integer")
    info.smem_bytes = raw_smem
    arch = meta.get("arch")
    if arch is not None:
        digits = arch[3:] if isinstance(arch, str) and arch.startswith("sm_") else ""
        if (not isinstance(arch, str) or not arch.startswith("sm_") or not digits
                or any(ch < "0" or ch > "9" for ch in digits)):
            raise CompileError(f"meta.json arch must look like 'sm_89': {arch!r}")
    if "args" not in meta:
        raise CompileError("meta.json is missing args")
    args = meta["args"]
    if not isinstance(args, list):
        raise CompileError("meta.json args must be a list")
    seen = set()
    for arg in args:
        if not isinstance(arg, dict):
            raise CompileError("each meta.json argument must be an object")
        name = arg.get("name")
        if not isinstance(name, str) or not name:
            raise CompileError("each meta.json argument needs a non-empty name")
        if name in seen:
            raise CompileError(f"meta.json has duplicate argument {name!r}")
        seen.add(name)
        if "shape" not in arg:
            raise CompileError(f"meta.json argument {name!r} is missing shape")
        raw_shape = arg["shape"]
        if not isinstance(raw_shape, (list, tuple)):
            raise CompileError(f"meta.json argument {name!r} shape must be a list")
        if any(isinstance(x, bool) or not isinstance(x, int) for x in raw_shape):
            raise CompileError(
                f"meta.json argument {name!r} shape must contain integers: {raw_shape!r}")
        if any(x < 0 for x in raw_shape):
            raise CompileError(
                f"meta.json argument {name!r} shape must be non-negative: {raw_shape!r}")
        if "dtype" not in arg:
            raise CompileError(f"meta.json argument {name!r} is missing dtype")
        dt = norm_dtype(arg["dtype"])
        check_dtype(dt, f"argument {name!r}")
        if "scalar" in arg and not isinstance(arg["scalar"], bool):
            raise CompileError(f"meta.json argument {name!r} scalar must be a boolean")
        info.shapes[name] = tuple(raw_shape)
        info.dtypes[name] = dt
        if arg.get("output"):
            info.outputs.append(name)
        if arg.get("scalar"):
            info.scalars.add(name)
        if "data" in arg and isinstance(arg["data"], list):
            info.data[name] = list(arg["data"])
    if "arg_order" not in meta:
        raise CompileError("meta.json is missing arg_order")
    order = meta["arg_order"]
    if not isinstance(order, list) or not all(isinstance(x, str) for x in order):
        raise CompileError("meta.json arg_order must be a list of argument names")
    duplicates = sorted({name for name in order if order.count(name) > 1})
    if duplicates:
        raise CompileError("meta.json arg_order has duplicate entries: " + ", ".join(duplicates))
    if seen and not order:
        raise CompileError("meta.json arg_order must list every argument")
    missing = sorted(seen - set(order))
    extra = sorted(set(order) - seen)
    if missing or extra:
        detail = []
        if missing:
            detail.append("missing " + ", ".join(missing))
        if extra:
            detail.append("unknown " + ", ".join(extra))
        raise CompileError("meta.json arg_order must name every argument (" + "; ".join(detail) + ")")
    info.arg_order = list(order)
    zo = meta.get("zero_outputs") or []
    if not isinstance(zo, list) or not all(isinstance(x, str) for x in zo):
        raise CompileError("meta.json zero_outputs must be a list of argument names")
    unknown = sorted(set(zo) - seen)
    if unknown:
        raise CompileError("meta.json zero_outputs names unknown arguments: " + ", ".join(unknown))
    info.zero_outputs = list(zo)
    return info
