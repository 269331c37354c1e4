"""``Lowerer``: Kernel IR + meta.json -> B200 launch plan.

The reference ``Lowerer`` (``ptxc/lower.py:36-108`` set-up, ``:549-595``
``compile``) validates meta.json, then walks the statement tree once and prints
PTX.  This ``Lowerer`` keeps the same constructor, the same validation and
error contract (``CompileError``; unexpected ``TypeError``/``KeyError``/...
re-raised as ``CompileError("invalid IR: ...")``, ``ptxc/lower.py:37-43`` and
``:549-555``), and the reference's launch guards (``ptxc/lower.py:736-825``),
but instead of emitting a generic walk it recognises which kernel family the
IR is and returns a launch plan for the hand-written sm_100a kernel of that
family in ``libemmyb200.so``.  An IR no family matches raises
``CompileError``: there is no generic or CPU fallback.

``compile()`` returns the plan as deterministic ASCII JSON (sorted keys, fixed
float formatting), which ``compile.py`` prints; ``plan()`` returns it as a
dict and ``ptxc.launch.run`` executes it.
"""

from __future__ import annotations

import json
import math

from .common import CompileError, iter_stmts, stmt_name
from .match_reduce import NoMatch, match_reduction
from .meta import read_meta

PLAN_FORMAT = "emmy-b200-plan/1"

def _has_block_collective(stmts) -> bool:
    """A block-wide combine or barrier anywhere below (``ptxc/lower.py:704-717``)."""
    return any(stmt_name(st) == "TreeHalve"
               or (stmt_name(st) == "Sync" and not getattr(st, "warp", False))
               for st in iter_stmts(stmts))


def _has_warp_collective(stmts) -> bool:
    """A warp shuffle or warp barrier anywhere below (``ptxc/lower.py:720-733``)."""
    return any(stmt_name(st) == "WarpShuffle"
               or (stmt_name(st) == "Sync" and getattr(st, "warp", False))
               for st in iter_stmts(stmts))


def _matchers():
    from .match_gemm import match_gemm
    from .match_attention import match_attention
    from .match_pointwise import match_pointwise
    return [("pointwise", match_pointwise), ("reduction", match_reduction),
            ("matmul", match_gemm), ("attention", match_attention)]


class Lowerer:
    def __init__(self, kernel_op, meta_kernel) -> None:
        try:
            self._init(kernel_op, meta_kernel)
        except CompileError:
            raise
        except (TypeError, AttributeError, KeyError, IndexError, ValueError, OverflowError) as exc:
            raise CompileError(f"invalid IR: {exc}") from exc

    def _init(self, kernel_op, meta_kernel) -> None:
        self.op = kernel_op
        self.name = kernel_op.name
        self.meta_raw = meta_kernel if meta_kernel is not None else {}
        self.meta = read_meta(self.meta_raw)
        body = tuple(kernel_op.body)
        tiles = [st for st in body if stmt_name(st) == "Tile"]
        if len(tiles) != 1:
            raise CompileError(f"expected exactly one Tile in {self.name!r}, found {len(tiles)}")
        for st in body:
            if stmt_name(st) not in ("Tile", "Smem"):
                raise CompileError(f"statement {stmt_name(st)} outside the Tile is not supported")
        self.tile = tiles[0]
        for st in iter_stmts(body):
            if stmt_name(st) not in ("Tile", "Loop", "StridedLoop", "Load", "Write", "Assign",
                                     "Accum", "Let", "Init", "Smem", "Cond", "Sync",
                                     "WarpShuffle", "TreeHalve", "CpAsyncCopy", "CpAsyncCommit",
                                     "CpAsyncWait", "ZeroPrologue"):
                raise CompileError(f"unsupported statement {stmt_name(st)}")
        self._check_launch()
        self._plan = None

    def _check_launch(self) -> None:
        """The reference's Tile guards (``ptxc/lower.py:736-783``)."""
        axes = []
        for axis in self.tile.axes:
            try:
                ext = int(axis.extent.value)
            except (AttributeError, TypeError, ValueError):
                raise CompileError(
                    f"Tile axis {axis.name!r} has no constant extent; static shapes only")
            axes.append((axis.name, ext))
        n = math.prod(e for _, e in axes) if axes else 1
        threads = math.prod(self.meta.block)
        launch = threads * math.prod(self.meta.grid)
        if n < launch:
            if n % threads and _has_block_collective(self.tile.body):
                raise CompileError(
                    f"block collective under a partial block: {n} tiles, "
                    f"{threads} threads per block, {launch} launched. "
                    "The gid guard would skip part of the barrier.")
            if n % 32 and _has_warp_collective(self.tile.body):
                raise CompileError(
                    f"warp collective under a partial warp: {n} tiles, "
                    f"{launch} launched. The full mask would include inactive lanes.")
        if n > launch:
            raise CompileError(
                f"meta.json launch of {launch} threads covers only part of the {n} Tile "
                "work items")
        self.tile_count = n

    def plan(self) -> dict:
        if self._plan is None:
            try:
                self._plan = self._build_plan()
            except CompileError:
                raise
            except (TypeError, AttributeError, KeyError, IndexError, ValueError,
                    OverflowError) as exc:
                raise CompileError(f"invalid IR: {exc}") from exc
        return self._plan

    def _build_plan(self) -> dict:
        reasons = []
        for fam, fn in _matchers():
            try:
                body = fn(self.op, self.tile, self.meta)
            except NoMatch as exc:
                reasons.append(f"{fam}: {exc}")
                continue
            return self._finish(body)
        raise CompileError(
            f"no B200 kernel family matches {self.name!r} (there is no generic fallback): "
            + "; ".join(reasons))

    def _finish(self, body: dict) -> dict:
        m = self.meta
        plan = {
            "format": PLAN_FORMAT,
            "entry": self.name,
            "arg_order": list(m.arg_order),
            "tensors": {name: {"dtype": m.dtypes[name], "shape": list(m.shapes[name])}
                        for name in m.arg_order},
            "outputs": [name for name in m.arg_order if name in m.outputs],
            "zero_outputs": list(m.zero_outputs),
            "meta_launch": {"grid": list(m.grid), "block": list(m.block),
                            "smem_bytes": m.smem_bytes},
            "tile_items": self.tile_count,
        }
        plan.update(body)
        return plan

    def compile(self) -> str:
        try:
            plan = self.plan()
        except CompileError:
            raise
        text = json.dumps(plan, sort_keys=True, indent=1, ensure_ascii=False) + "\n"
        if not text.isascii():
            raise CompileError("launch plan must be ASCII")
        return text
