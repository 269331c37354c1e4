"""TEST INFRASTRUCTURE ONLY -- torch-CPU evaluation of a Kernel IR.

This is the parity oracle and the timed CPU baseline ("torch-CPU evaluation of
the IR").  Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU
legs may import it; the product path (``compile.py`` -> ``ptxc`` -> the CUDA
library) never does.

It restates, statement by statement, the semantics the reference compiler
gives each IR statement when it lowers a KernelOp to PTX, and runs them over
every thread of the launch at once: one tensor lane per flattened work id
``gid``.  Lanes advance in lockstep, which is a legal schedule for
barrier-synchronised code, so ``Sync`` needs no action.

Semantics followed (reference file:line):

* launch and Tile decode: ``gid = ctaid.x*ntid.x + tid.x`` (``ptxc/lower.py:828-848``);
  ``idx_i = (gid / suffix_i) % extent_i`` with ``suffix_i`` the product of the
  later extents, a single axis binds ``gid`` itself, lanes with ``gid >= N``
  are inactive (``ptxc/lower.py:736-825``).
* flat index: row-major strides over the buffer shape for as many
  coordinates as given; a lone coordinate is already flat
  (``ptxc/common.py:398-415``, ``ptxc/memory.py:150-186``).
* ``Accum``: ``acc = op(base if base else acc, value)``; accumulators are
  seeded at the entry of the loop instance named by ``axes[0]`` unless an
  ``Init`` names them, top-level ones at kernel entry, others lazily on first
  fold (``ptxc/stmts.py:564-611``, ``ptxc/lower.py:524-546,651-677``,
  ``ptxc/common.py:87-112``); seeds are ``add->0``, ``max->-1e30``,
  ``min->1e30`` (``ptxc/ops.py:67-75``).  A half accumulator is rounded
  back to f16 after every fold (``ptxc/stmts.py:589-594``).
* ``StridedLoop``: ``for a in start..end step s`` per lane (``ptxc/stmts.py:728-773``);
  ``Loop``: ``for a in 0..extent`` (``ptxc/stmts.py:663-725``).
* ``WarpShuffle``: XOR butterfly for ``offset = length/2 .. 1`` then the
  combine statements (``ptxc/stmts.py:1441-1492``).
* ``TreeHalve``: for ``s = length/2 .. 1`` threads ``tid < s`` fold slot
  ``tid+s`` into slot ``tid``; afterwards every thread reads slot 0
  (``ptxc/stmts.py:1495-1568``).
* ``Load``/``Write``: f16 loads widen to f32; a write converts to the
  destination dtype (``ptxc/stmts.py:434-487``); atomic writes add
  (``red.global.add``).
* ``CpAsyncCopy``: ``nbytes`` consecutive elements from ``src[src_index]`` to
  ``smem[smem_index (+ lane_index over (.., cols))]`` (``ptxc/stmts.py:1590-1623``).
  A coordinate written ``None + e`` in a copy inside a ``StridedLoop`` stands
  for ``loop_var + step + e`` (the next pipeline stage; see the prefetch
  copies of the reference fixture ``tests/variants/v_m_256``); source reads
  past the end of the buffer are skipped, since their stage is never used.
* elementwise ops: the f32 spellings of ``ptxc/expr.py:880-1089``
  (``exp`` is ``2^(x*log2 e)``, ``reciprocal`` is ``1/x`` rounded once,
  ``maximum`` is ``max``, ``add``/``sub``/``mul`` rounded per op).  Values
  are float32 tensors for f32/f16 work and float64 for f64 work.
"""

from __future__ import annotations

import math
import sys
from pathlib import Path

import numpy as np
import torch

_PKG = Path(__file__).resolve().parent.parent / "emmy-ptx-compiler-submission_b200"
if str(_PKG) not in sys.path:
    sys.path.insert(0, str(_PKG))

from emmy_ir.nodes import (  # noqa: E402
    BinaryExpr, Builtin, CastExpr, Dim, Literal, TernaryExpr, Var, dtype_name, iter_stmts,
)

# u16 / u32 / u64 buffers are held as the signed tensor of the same width (the
# same bits; ``run_ir`` views them so) and widened with a mask on load
TORCH_DT = {"f32": torch.float32, "f16": torch.float16, "f64": torch.float64,
            "i32": torch.int32, "i64": torch.int64, "u8": torch.uint8, "i8": torch.int8,
            "i16": torch.int16, "u16": torch.int16, "u32": torch.int32, "u64": torch.int64,
            "bool": torch.bool}
NP_DT = {"f32": np.float32, "f16": np.float16, "f64": np.float64, "i32": np.int32,
         "i64": np.int64, "u8": np.uint8, "i8": np.int8, "i16": np.int16, "u16": np.uint16,
         "u32": np.uint32, "u64": np.uint64, "bool": np.bool_}
INT_DT = {"i8", "u8", "i16", "u16", "i32", "u32", "i64", "u64"}
_UNSIGNED_MASK = {"u16": 0xFFFF, "u32": 0xFFFFFFFF}
_SIGNED_VIEW = {np.dtype(np.uint16): np.int16, np.dtype(np.uint32): np.int32,
                np.dtype(np.uint64): np.int64}

IDENTITY = {"add": 0.0, "sum": 0.0, "multiply": 1.0, "prod": 1.0,
            "maximum": -1e30, "amax": -1e30, "minimum": 1e30}


class OracleError(RuntimeError):
    pass


def _op_name(op) -> str:
    return getattr(op, "name", str(op))


def _strides(shape, ncoords):
    shape = tuple(int(s) for s in shape)
    if ncoords <= 1 or not shape:
        return [1] * ncoords
    out = []
    for i in range(ncoords):
        s = 1
        for d in shape[i + 1:]:
            s *= d
        out.append(s)
    return out


def _compute_kind(dt: str) -> str:
    return "f64" if dt == "f64" else ("f32" if dt in ("f32", "f16") else dt)


class IRInterpreter:
    """Run one KernelOp under its meta launch over CPU tensors.

    ``buffers`` maps every argument name to a 1-D CPU tensor of the argument's
    dtype and ``prod(shape)`` elements (outputs must already hold their
    initial contents; the caller zeroes them as the reference harness does).
    ``blocks=(b0, b1)`` restricts the run to a range of thread blocks, which
    ``bench.py`` uses to time a bounded sample of a large launch.
    """

    def __init__(self, kernel_op, meta: dict, buffers: dict, blocks=None):
        self.op = kernel_op
        self.meta = meta
        self.buffers = buffers
        self.shapes = {a["name"]: tuple(a["shape"]) for a in meta["args"]}
        self.dtypes = {a["name"]: a["dtype"] for a in meta["args"]}
        self.threads = int(np.prod(meta["block"]))
        grid = int(np.prod(meta["grid"]))
        b0, b1 = (0, grid) if blocks is None else blocks
        self.gid = torch.arange(b0 * self.threads, b1 * self.threads, dtype=torch.int64)
        self.L = self.gid.numel()
        self.tid = self.gid % self.threads
        self.blk = self.gid // self.threads - b0
        self.nblk = b1 - b0
        self.env = {}          # name -> (tensor, kind)
        self.axes = {}         # axis name -> int64 tensor or int
        self.smem = {}         # name -> (tensor [nblk, n], dtype, extents)
        self.inits = set()
        self.loop_stack = []   # (axis name, var tensor, step)
        for st in iter_stmts(kernel_op.body):
            if type(st).__name__ == "Init":
                self.inits.add(st.name)

    # -- entry ---------------------------------------------------------------

    def run(self):
        body = self.op.body
        tiles = [s for s in body if type(s).__name__ == "Tile"]
        if len(tiles) != 1:
            raise OracleError("expected exactly one Tile at the top of the kernel")
        pre = [s for s in body if type(s).__name__ != "Tile"]
        mask = torch.ones(self.L, dtype=torch.bool)
        self._seed_top(body)
        self._walk(pre, mask)
        tile = tiles[0]
        axes = [(a.name, int(a.extent.value)) for a in tile.axes]
        n = 1
        for _, e in axes:
            n *= e
        suffix = [1] * len(axes)
        for i in range(len(axes) - 2, -1, -1):
            suffix[i] = suffix[i + 1] * axes[i + 1][1]
        if len(axes) == 1 and axes[0][1] > 1:
            self.axes[axes[0][0]] = self.gid
        else:
            for (name, ext), suf in zip(axes, suffix):
                self.axes[name] = (self.gid // suf) % ext
        active = self.gid < n
        self._walk(tile.body, active)

    def _seed_top(self, body):
        seen = {}
        for st in iter_stmts(body):
            if type(st).__name__ == "Accum":
                seen.setdefault(st.name, st)
        for name, st in seen.items():
            if name in self.inits or tuple(st.axes or ()):
                continue
            self._seed(st, torch.ones(self.L, dtype=torch.bool))

    # -- helpers ---------------------------------------------------------------

    def _set(self, name, value, kind, mask):
        if isinstance(value, torch.Tensor) and value.dim() == 0:
            value = value.expand(self.L)
        old = self.env.get(name)
        if old is not None and not bool(mask.all()):
            ov = old[0]
            if ov.dtype != value.dtype:
                ov = ov.to(value.dtype)
            if ov.dim() == 0:
                ov = ov.expand(self.L)
            value = torch.where(mask, value, ov)
        self.env[name] = (value, kind)

    def _const(self, v, kind):
        if kind == "f64":
            return torch.tensor(float(v), dtype=torch.float64)
        if kind in ("f32", "f16"):
            return torch.tensor(float(v), dtype=torch.float32)
        if kind == "pred":
            return torch.tensor(bool(v))
        return torch.tensor(int(v), dtype=torch.int64)

    def _value(self, name):
        if isinstance(name, (int, float)) and not isinstance(name, bool):
            return self._const(name, "f32" if isinstance(name, float) else "i64"), \
                ("f32" if isinstance(name, float) else "i64")
        if name in self.env:
            return self.env[name]
        if name in self.axes:
            return self._as_tensor(self.axes[name]), "i64"
        if name in ("lane", "lane_id"):
            return self.tid % 32, "i64"
        if name in ("warp", "warp_id"):
            return self.tid // 32, "i64"
        if name in ("tid", "thread_id", "thread_idx.x"):
            return self.tid, "i64"
        raise OracleError(f"unknown SSA value {name!r}")

    def _as_tensor(self, v):
        if isinstance(v, torch.Tensor):
            return v
        return torch.tensor(int(v), dtype=torch.int64)

    def _seed(self, st, mask):
        dt = dtype_name(st.dtype)
        kind = _compute_kind(dt)
        ident = IDENTITY.get(_op_name(st.op), 0.0)
        v = self._const(ident, kind)
        if dt == "f16":
            v = v.to(torch.float16).to(torch.float32)
        self._set(st.name, v.expand(self.L).clone(), kind, mask)

    def _seed_loop(self, loop, mask):
        axis = loop.axis.name
        found = []

        def walk(stmts, shadowed=False):
            for s in stmts:
                nm = type(s).__name__
                if nm == "Accum" and not shadowed:
                    ax = tuple(s.axes or ())
                    if ax and ax[0] == axis and s.name not in self.inits:
                        found.append(s)
                child_sh = shadowed or (nm in ("Loop", "StridedLoop") and s.axis.name == axis)
                for attr in ("body", "else_body"):
                    ch = getattr(s, attr, None)
                    if isinstance(ch, (tuple, list)) and ch:
                        walk(ch, child_sh)

        walk(loop.body)
        done = set()
        for s in found:
            if s.name not in done:
                done.add(s.name)
                self._seed(s, mask)

    # -- index expressions -------------------------------------------------------

    def idx(self, e):
        """An integer expression over axes, loop variables and builtins (int64)."""
        if e is None:
            raise OracleError("None in an index expression outside a pipelined copy")
        if isinstance(e, Dim):
            return torch.tensor(int(e.value), dtype=torch.int64)
        if isinstance(e, (int,)) and not isinstance(e, bool):
            return torch.tensor(e, dtype=torch.int64)
        if isinstance(e, Literal):
            return torch.tensor(int(e.value), dtype=torch.int64)
        if isinstance(e, (Var, Builtin)):
            if e.name in self.axes:
                return self._as_tensor(self.axes[e.name])
            v, kind = self._value(e.name)
            if kind in ("f32", "f64", "f16"):
                return torch.trunc(v).to(torch.int64)
            return v.to(torch.int64)
        if isinstance(e, BinaryExpr):
            if e.left is None or e.right is None:
                if not self.loop_stack:
                    raise OracleError("None operand outside a loop")
                _, var, step = self.loop_stack[-1]
                nxt = var + step
                other = e.right if e.left is None else e.left
                return self._ibin(e.op, nxt, self.idx(other)) if e.left is None \
                    else self._ibin(e.op, self.idx(other), nxt)
            return self._ibin(e.op, self.idx(e.left), self.idx(e.right))
        if isinstance(e, TernaryExpr):
            return torch.where(self.pred(e.cond), self.idx(e.if_true), self.idx(e.if_false))
        if isinstance(e, CastExpr):
            return self.idx(e.expr)
        raise OracleError(f"unsupported index expression {type(e).__name__}")

    @staticmethod
    def _ibin(op, a, b):
        if op in ("+", "add"):
            return a + b
        if op in ("-", "subtract"):
            return a - b
        if op in ("*", "multiply"):
            return a * b
        if op in ("/", "//", "divide", "floor_divide"):
            # s32 division truncates toward zero (div.s32); indices are non-negative
            return torch.div(a, b, rounding_mode="trunc")
        if op in ("%", "mod", "remainder"):
            return torch.fmod(a, b)
        if op in ("<<", "left_shift"):
            return a << b
        if op in (">>", "right_shift"):
            return a >> b
        if op == "&":
            return a & b
        if op == "|":
            return a | b
        if op == "^":
            return a ^ b
        raise OracleError(f"unsupported index op {op!r}")

    def pred(self, e):
        if isinstance(e, BinaryExpr):
            op = e.op
            rel = {"<": torch.lt, "<=": torch.le, ">": torch.gt, ">=": torch.ge,
                   "==": torch.eq, "!=": torch.ne}.get(op)
            if rel is not None:
                return rel(self.idx(e.left), self.idx(e.right))
            if op in ("and", "&&"):
                return self.pred(e.left) & self.pred(e.right)
            if op in ("or", "||"):
                return self.pred(e.left) | self.pred(e.right)
        if isinstance(e, Var):
            v, kind = self._value(e.name)
            return v != 0 if kind != "pred" else v
        raise OracleError(f"unsupported predicate {e!r}")

    def flat(self, index, shape):
        if index is None or len(index) == 0:
            return torch.tensor(0, dtype=torch.int64)
        if len(index) == 1:
            return self.idx(index[0])
        acc = None
        for coord, stride in zip(index, _strides(shape, len(index))):
            t = self.idx(coord) * stride
            acc = t if acc is None else acc + t
        return acc

    # -- statements --------------------------------------------------------------

    def _walk(self, stmts, mask):
        for st in stmts:
            getattr(self, "s_" + type(st).__name__)(st, mask)

    def s_Tile(self, st, mask):
        raise OracleError("nested Tile")

    def s_Smem(self, st, mask):
        if st.name in self.smem:
            return
        dt = dtype_name(st.dtype)
        n = int(np.prod([int(x) for x in st.extents])) if st.extents else 1
        self.smem[st.name] = (torch.zeros((self.nblk, n), dtype=TORCH_DT[dt]), dt,
                              tuple(int(x) for x in st.extents))

    def s_Sync(self, st, mask):
        pass

    def s_CpAsyncCommit(self, st, mask):
        pass

    def s_CpAsyncWait(self, st, mask):
        pass

    def s_Let(self, st, mask):
        dt = dtype_name(st.dtype)
        kind = _compute_kind(dt)
        value = getattr(st.value, "value", st.value)
        if dt in INT_DT and isinstance(value, float):
            # a float literal in an integer Let: its f32 value, truncated (cvt.rzi.s64.f32)
            value = int(_rzi_s64(torch.tensor([value], dtype=torch.float32))[0])
        self._set(st.name, self._const(value, kind).expand(self.L), kind, mask)

    def s_Init(self, st, mask):
        dt = dtype_name(st.dtype)
        kind = _compute_kind(dt)
        value = getattr(st.identity, "value", st.identity)
        self._set(st.name, self._const(value, kind).expand(self.L).clone(), kind, mask)

    def _gather(self, name, flat, mask):
        """Read one element per lane from a global or shared buffer."""
        flat = flat.expand(self.L) if flat.dim() == 0 else flat
        if name in self.smem:
            buf, dt, _ = self.smem[name]
            n = buf.shape[1]
            safe = torch.where(mask & (flat >= 0) & (flat < n), flat, torch.zeros_like(flat))
            return buf[self.blk, safe], dt
        buf = self.buffers[name]
        dt = self.dtypes[name]
        n = buf.numel()
        if n == 0:
            raise OracleError(f"load from empty buffer {name!r}")
        bad = mask & ((flat < 0) | (flat >= n))
        if bool(bad.any()):
            raise OracleError(f"out-of-bounds load from {name!r}")
        safe = torch.where(mask, flat, torch.zeros_like(flat))
        return buf[safe], dt

    def s_Load(self, st, mask):
        if st.input in self.smem:
            shape = self.smem[st.input][2]
        else:
            shape = self.shapes[st.input]
        base = self.flat(st.index, shape)
        for i, name in enumerate(st.names):
            raw, dt = self._gather(st.input, base + i, mask)
            kind = _compute_kind(dt)
            if kind == "f32":
                raw = raw.to(torch.float32)
            elif kind == "f64":
                raw = raw.to(torch.float64)
            else:
                # ld.s8 / ld.u8 ... widen with sign or zero extension
                raw = raw.to(torch.int64)
                if dt in _UNSIGNED_MASK:
                    raw = raw & _UNSIGNED_MASK[dt]
            self._set(name, raw, kind, mask)

    def _convert(self, v, kind, dt):
        """The store conversion (reference ``_cast_reg``, ptxc/expr.py:233-280)."""
        tdt = TORCH_DT[dt]
        if dt in ("f32", "f16", "f64"):
            if kind not in ("f32", "f64", "f16", "pred"):
                # an s64 value: cvt.rn.f64.s64, or cvt.rn.f32.s64 (then cvt.rn.f16.f32)
                if dt == "f64":
                    return v.to(torch.float64)
                return v.to(torch.float32).to(tdt)
            return v.to(tdt)
        if kind in ("f32", "f64"):
            v = _rzi_s64(v)
        # the low bits of the s64 value (st.u8 / cvt.s32.s64 ...)
        return v.to(torch.int64).to(tdt)

    def s_Write(self, st, mask):
        if st.output in self.smem:
            buf, dt, ext = self.smem[st.output]
            base = self.flat(st.index, ext)
            for i, vname in enumerate(st.values):
                v, kind = self._value(vname)
                v = v.expand(self.L) if v.dim() == 0 else v
                f = (base + i)
                f = f.expand(self.L) if f.dim() == 0 else f
                if getattr(st, "swizzle", "NONE") not in (None, "NONE"):
                    f = _swizzle(f, st.swizzle)
                m = mask
                buf[self.blk[m], f[m]] = self._convert(v[m], kind, dt)
            return
        buf = self.buffers[st.output]
        dt = self.dtypes[st.output]
        base = self.flat(st.index, self.shapes[st.output])
        for i, vname in enumerate(st.values):
            v, kind = self._value(vname)
            v = v.expand(self.L) if v.dim() == 0 else v
            f = base + i
            f = f.expand(self.L) if f.dim() == 0 else f
            m = mask
            idx = f[m]
            if idx.numel() and (int(idx.min()) < 0 or int(idx.max()) >= buf.numel()):
                raise OracleError(f"out-of-bounds write to {st.output!r}")
            val = self._convert(v[m], kind, dt)
            if st.atomic:
                if dt == "f16":
                    # red.global.add.f16 rounds each add; emulate in f32 then round
                    acc = buf.to(torch.float32)
                    acc.index_put_((idx,), val.to(torch.float32), accumulate=True)
                    buf.copy_(acc.to(torch.float16))
                else:
                    buf.index_put_((idx,), val, accumulate=True)
            else:
                buf[idx] = val

    def s_Assign(self, st, mask):
        opname = _op_name(st.op)
        vals = [self._value(a) for a in st.args]
        dt = dtype_name(st.dtype) if st.dtype is not None else None
        kinds = [k for _, k in vals]
        if dt is None or dt in INT_DT or dt == "bool" or any(k in INT_DT or k == "pred"
                                                              for k in kinds):
            res = _int_assign(opname, dt, vals)
            if res is not None:
                self._set(st.name, res[0], res[1], mask)
                return
        if dt is None:
            kind = "f64" if "f64" in kinds else ("f32" if any(k in ("f32", "f16") for k in kinds) else kinds[0])
        else:
            kind = _compute_kind(dt)
        out = _elementwise(opname, [v for v, _ in vals], kinds, kind)
        if isinstance(out, tuple):
            out, kind = out
        if dt == "f16":
            out = out.to(torch.float16).to(torch.float32)
        self._set(st.name, out, kind, mask)

    def s_Accum(self, st, mask):
        opname = _op_name(st.op)
        dt = dtype_name(st.dtype)
        kind = _compute_kind(dt)
        if st.name not in self.env:
            self._seed(st, mask)
        left = self._value(st.base)[0] if st.base is not None else self.env[st.name][0]
        right = self._value(st.value)[0]
        out = _elementwise(opname, [left, right], [kind, kind], kind)
        if isinstance(out, tuple):
            out = out[0]
        if dt == "f16":
            out = out.to(torch.float16).to(torch.float32)
        self._set(st.name, out, kind, mask)

    def s_Cond(self, st, mask):
        p = self.pred(st.cond)
        p = p.expand(self.L) if p.dim() == 0 else p
        m1 = mask & p
        if bool(m1.any()):
            self._walk(st.body, m1)
        if st.else_body:
            m2 = mask & ~p
            if bool(m2.any()):
                self._walk(st.else_body, m2)

    def s_Loop(self, st, mask):
        name = st.axis.name
        ext = int(st.axis.extent.value)
        saved = self.axes.get(name)
        self._seed_loop(st, mask)
        for i in range(ext):
            var = torch.tensor(i, dtype=torch.int64)
            self.axes[name] = var
            self.loop_stack.append((name, var, 1))
            self._walk(st.body, mask)
            self.loop_stack.pop()
        if saved is None:
            self.axes.pop(name, None)
        else:
            self.axes[name] = saved

    def s_StridedLoop(self, st, mask):
        name = st.axis.name
        start = self.idx(st.start)
        start = start.expand(self.L) if start.dim() == 0 else start
        end = self.idx(st.end if st.end is not None else st.axis.extent)
        step = int(st.step.value)
        if step <= 0:
            raise OracleError("StridedLoop step must be positive")
        saved = self.axes.get(name)
        self._seed_loop(st, mask)
        span = (end - start).clamp(min=0)
        trips = torch.div(span + step - 1, step, rounding_mode="floor")
        tmax = int(trips[mask].max()) if bool(mask.any()) else 0
        for t in range(tmax):
            var = start + t * step
            m = mask & (var < end)
            self.axes[name] = var
            self.loop_stack.append((name, var, step))
            self._walk(st.body, m)
            self.loop_stack.pop()
        if saved is None:
            self.axes.pop(name, None)
        else:
            self.axes[name] = saved

    def s_WarpShuffle(self, st, mask):
        length = int(st.length)
        lane = self.tid % 32
        offset = length // 2
        while offset >= 1:
            partner_tid = (self.tid - lane) + (lane ^ offset)
            if bool((partner_tid >= self.threads).any()):
                raise OracleError("shuffle partner outside the block")
            # lanes are laid out block-major, so the partner's lane index is
            # this lane's index plus the tid difference
            pidx = torch.arange(self.L) + (partner_tid - self.tid)
            for s, sb in zip(st.state, st.state_b):
                v, kind = self.env[s]
                v = v.expand(self.L) if v.dim() == 0 else v
                self._set(sb, v[pidx], kind, mask)
            self._walk(st.combine_states, mask)
            offset //= 2

    def s_TreeHalve(self, st, mask):
        if st.inner:
            raise OracleError("TreeHalve with an inner offset is not restated")
        length = int(st.length)
        tid = self._value(st.tid_var)[0]
        tid = tid.expand(self.L) if tid.dim() == 0 else tid
        s = length // 2
        while s >= 1:
            m = mask & (tid < s)
            for state, sb, bufname in zip(st.state, st.state_b, st.bufs):
                buf, dt, _ = self.smem[bufname]
                kind = _compute_kind(dt)
                a = buf[self.blk, torch.where(m, tid, torch.zeros_like(tid))]
                b = buf[self.blk, torch.where(m, tid + s, torch.zeros_like(tid))]
                conv = torch.float64 if kind == "f64" else torch.float32
                self._set(state, a.to(conv), kind, m)
                self._set(sb, b.to(conv), kind, m)
            self._walk(st.combine_states, m)
            for state, bufname in zip(st.state, st.bufs):
                buf, dt, _ = self.smem[bufname]
                v, kind = self.env[state]
                buf[self.blk[m], tid[m]] = self._convert(v[m], kind, dt)
            s //= 2
        for state, bufname in zip(st.state, st.bufs):
            buf, dt, _ = self.smem[bufname]
            kind = _compute_kind(dt)
            conv = torch.float64 if kind == "f64" else torch.float32
            self._set(state, buf[self.blk, 0].to(conv), kind, mask)

    def s_CpAsyncCopy(self, st, mask):
        buf, dt, ext = self.smem[st.smem]
        esize = torch.empty((), dtype=TORCH_DT[dt]).element_size()
        count = int(st.nbytes) // esize
        dst = self.flat(st.smem_index, ext)
        if st.lane_index is not None:
            cols = ext[-1]
            dst = dst + self.flat(st.lane_index, (0, cols))
            if getattr(st, "swizzle", "NONE") not in (None, "NONE"):
                dst = _swizzle(dst, st.swizzle)
        src = self.flat(st.src_index, self.shapes[st.src])
        dst = dst.expand(self.L) if dst.dim() == 0 else dst
        src = src.expand(self.L) if src.dim() == 0 else src
        sbuf = self.buffers[st.src]
        for i in range(count):
            s = src + i
            ok = mask & (s >= 0) & (s < sbuf.numel())
            if not bool(ok.any()):
                continue
            buf[self.blk[ok], (dst + i)[ok]] = sbuf[s[ok]].to(buf.dtype)

    def s_ZeroPrologue(self, st, mask):
        buf = self.buffers[st.dst]
        nbytes = int(st.words) * 4
        view = buf.view(torch.uint8)
        view[:nbytes] = 0


def _swizzle(flat, mode):
    base, _, sh = str(mode).partition("@")
    shift, msk = {"B32": (1, 1), "B64": (1, 3), "B128": (1, 7)}.get(base, (0, 0))
    if sh:
        shift = int(sh)
    if not msk:
        return flat
    return flat ^ (((flat >> shift) & msk) << 3)


def _f(v, kind):
    return v


def _rn32(x64):
    """Round a float64 result to float32 (one rounding of the exact value when
    float64 holds it to 2*24+2 bits, as for +, -, *, /, sqrt)."""
    return x64.to(torch.float32)


def _fma_rn(a, b, c, tdt):
    """a*b + c rounded once (fma.rn): exact rational sum, then one rounding.

    float64: ``Fraction.__float__`` rounds correctly.  float32: the float64
    nearest is moved to its odd neighbour when inexact (round-to-odd at 53
    bits), after which rounding to 24 bits is correct.
    """
    from fractions import Fraction
    a, b, c = torch.broadcast_tensors(a.to(tdt), b.to(tdt), c.to(tdt))
    av, bv, cv = (t.contiguous().reshape(-1).double().tolist() for t in (a, b, c))
    out = []
    for x, y, z in zip(av, bv, cv):
        if not (math.isfinite(x) and math.isfinite(y) and math.isfinite(z)):
            out.append(x * y + z)
            continue
        exact = Fraction(x) * Fraction(y) + Fraction(z)
        d = float(exact)
        if tdt == torch.float32 and Fraction(d) != exact and math.isfinite(d):
            if np.frombuffer(np.float64(d).tobytes(), np.int64)[0] & 1 == 0:
                d = float(np.nextafter(d, math.inf if exact > Fraction(d) else -math.inf))
        out.append(d)
    return torch.tensor(out, dtype=torch.float64).reshape(a.shape).to(tdt)


# ---------------------------------------------------------------------------
# Integer Assigns, as the reference lowers them (ptxc/stmts.py:509-560,
# ptxc/expr.py:157-165, 211-223, 697-716, 815-877, ptxc/ops.py:98-117): every
# operand becomes an s64 value (cvt.s64.<int type> widens; cvt.rzi.s64.<float
# type> truncates a float toward zero, saturating, NaN to -2^63), the op runs on
# s64 (add / sub / mul.lo wrap modulo 2^64, div.s64 / rem.s64 truncate toward
# zero, max / min and the comparisons are signed), a comparison or
# and / or / not gives a predicate (``bitwise_and`` / ``bitwise_or`` included:
# the reference sends them down its predicate path), ``where`` selects s64
# values.  Shifts take the low 32 bits of the count as unsigned (the PTX
# operand type) with shl.b64 / shr.s64 semantics past 63.

_INT_OPS = {"add", "sum", "subtract", "sub", "multiply", "prod", "divide", "floor_divide",
            "true_divide", "remainder", "mod", "left_shift", "right_shift", "bitwise_xor",
            "maximum", "amax", "minimum"}
_CMP_OPS = {"equal": "eq", "eq": "eq", "not_equal": "ne", "ne": "ne", "greater": "gt",
            "gt": "gt", "less": "lt", "lt": "lt", "greater_equal": "ge", "ge": "ge",
            "less_equal": "le", "le": "le"}
_BOOL_BINARY = {"bitwise_and", "logical_and", "and", "bitwise_or", "logical_or", "or"}
_BOOL_NOT = {"bitwise_not", "logical_not", "not"}
_I64_MIN, _I64_MAX = -(1 << 63), (1 << 63) - 1


def _rzi_s64(v):
    """cvt.rzi.s64.f32 / .f64: toward zero, clamped to the s64 range, NaN -> -2^63
    (the B200 running the reference's own PTX gives that)."""
    a = v.double().numpy() if isinstance(v, torch.Tensor) else np.asarray(v, np.float64)
    with np.errstate(invalid="ignore"):
        t = np.trunc(a)
    out = np.full(a.shape, _I64_MIN, np.int64)                 # NaN stays here
    inside = np.isfinite(t) & (t >= -9.223372036854775808e18) & (t < 9.223372036854775808e18)
    out[inside] = t[inside].astype(np.int64)
    out[t >= 9.223372036854775808e18] = _I64_MAX
    out[t < -9.223372036854775808e18] = _I64_MIN
    return torch.from_numpy(out)


def _s64_operand(v, kind):
    """The reference's ``iexpr_operand`` / ``_to_s64`` for one value."""
    if kind == "pred":
        raise OracleError("a predicate used as an integer operand")
    if kind in ("f32", "f64", "f16"):
        return _rzi_s64(v)
    return v.to(torch.int64)


def _pred_operand(v, kind):
    """The reference's ``pred_operand``: a predicate, else v != 0 (unordered for floats)."""
    if kind == "pred":
        return v.to(torch.bool)
    return v != 0


def _int_binary(op, a, b):
    a, b = torch.broadcast_tensors(a.to(torch.int64), b.to(torch.int64))
    x = a.contiguous().numpy()
    y = b.contiguous().numpy()
    ux, uy = x.view(np.uint64), y.view(np.uint64)
    if op in ("add", "sum"):
        r = (ux + uy).view(np.int64)
    elif op in ("subtract", "sub"):
        r = (ux - uy).view(np.int64)
    elif op in ("multiply", "prod"):
        r = (ux * uy).view(np.int64)
    elif op in ("divide", "floor_divide", "true_divide", "remainder", "mod"):
        if (y == 0).any():
            raise OracleError("integer division by zero (div.s64 leaves it unspecified)")
        if ((x == _I64_MIN) & (y == -1)).any():
            raise OracleError("s64 division overflow (div.s64 leaves it unspecified)")
        q = np.floor_divide(x, y)
        rem = x - q * y
        q = q + ((rem != 0) & ((x < 0) != (y < 0)))            # toward zero
        if op in ("remainder", "mod"):
            r = (ux - (q.view(np.uint64) * uy)).view(np.int64)
        else:
            r = q
    elif op in ("left_shift", "right_shift"):
        c = (uy & np.uint64(0xFFFFFFFF)).astype(np.uint64)
        cc = np.minimum(c, np.uint64(63))
        if op == "left_shift":
            r = np.where(c >= 64, np.uint64(0), ux << cc).view(np.int64)
        else:
            r = np.where(c >= 64, np.where(x < 0, -1, 0), x >> cc.astype(np.int64))
    elif op == "bitwise_xor":
        r = x ^ y
    elif op in ("maximum", "amax"):
        r = np.maximum(x, y)
    else:
        r = np.minimum(x, y)
    return torch.from_numpy(np.ascontiguousarray(r, dtype=np.int64))


def _int_assign(opname, dt, vals):
    """One Assign the reference lowers on its integer / predicate paths, or
    None when it lowers it as float arithmetic.  Returns (tensor, kind)."""
    kinds = [k for _, k in vals]
    ref_dt = dt if dt is not None else kinds[0]      # ``_infer_kind``: the first argument's
    floats = ("f32", "f64", "f16")
    if ref_dt == "bool" or opname in _CMP_OPS or opname in _BOOL_BINARY:
        if opname in _BOOL_BINARY:
            return _pred_operand(*vals[0]) & _pred_operand(*vals[1]) if "and" in opname else \
                _pred_operand(*vals[0]) | _pred_operand(*vals[1]), "pred"
        if opname in _BOOL_NOT:
            return ~_pred_operand(*vals[0]), "pred"
        if opname not in _CMP_OPS:
            raise OracleError(f"unsupported boolean op {opname!r}")
        if any(k in floats for k in kinds[:2]):
            return None
        a, b = _s64_operand(*vals[0]), _s64_operand(*vals[1])
        rel = _CMP_OPS[opname]
        return {"eq": a == b, "ne": a != b, "gt": a > b, "lt": a < b, "ge": a >= b,
                "le": a <= b}[rel], "pred"
    if opname == "where":
        if ref_dt in floats or kinds[1] in floats or kinds[2] in floats:
            return None
        c = _pred_operand(*vals[0])
        return torch.where(c, _s64_operand(*vals[1]), _s64_operand(*vals[2])), "i64"
    if ref_dt in floats:
        return None
    if opname in ("copy", "pad", "bitcast"):
        return vals[0][0].clone(), vals[0][1]
    if opname not in _INT_OPS:
        raise OracleError(f"unsupported integer op {opname!r}")
    return _int_binary(opname, _s64_operand(*vals[0]), _s64_operand(*vals[1])), "i64"


def _elementwise(opname, args, kinds, kind):
    """One elementwise op in the compute kind (f32 or f64 tensors, int64 or bool)."""
    fl = kind in ("f32", "f64")
    tdt = torch.float64 if kind == "f64" else torch.float32
    if fl:
        args = [a.to(tdt) if a.dtype != tdt and a.dtype != torch.bool else a for a in args]
    a = args[0] if args else None
    b = args[1] if len(args) > 1 else None
    if opname in ("add", "sum"):
        return a + b
    if opname in ("subtract", "sub"):
        return a - b
    if opname in ("multiply", "prod"):
        return a * b
    if opname in ("divide", "true_divide", "divide_rn_f32"):
        if kind == "f32":
            return _rn32(a.double() / b.double())
        return a / b if fl else torch.div(a, b, rounding_mode="trunc")
    if opname in ("maximum", "amax", "max"):
        return torch.maximum(a, b)
    if opname in ("minimum", "min"):
        return torch.minimum(a, b)
    if opname == "fma":
        return _fma_rn(a, b, args[2], tdt)
    if opname in ("exp", "exp_fast"):
        if kind == "f64":
            return torch.exp(a)
        return torch.exp2(a * torch.tensor(1.4426950408889634, dtype=torch.float32))
    if opname == "exp2":
        return torch.exp2(a)
    if opname == "log":
        return torch.log(a)
    if opname == "sqrt":
        # sqrt.rn is correctly rounded; torch's vectorised CPU sqrt is not
        # always (float32 and float64), numpy's is
        return torch.from_numpy(np.sqrt(a.contiguous().numpy()))
    if opname == "rsqrt":
        return torch.rsqrt(a)
    if opname == "reciprocal":
        return _rn32(1.0 / a.double()) if kind == "f32" else torch.reciprocal(a)
    if opname == "relu":
        return torch.clamp_min(a, 0)
    if opname in ("copy", "pad", "bitcast"):
        return a.clone()
    if opname in ("negative", "negate"):
        return -a
    if opname in ("abs", "fabs"):
        return torch.abs(a)
    if opname == "tanh":
        return torch.tanh(a)
    if opname == "sigmoid":
        return torch.sigmoid(a)
    if opname == "pow":
        return torch.pow(a, b)
    # the rest of the reference's float op table (ptxc/expr.py:899-1075)
    if opname == "log2":
        return torch.log2(a)
    if opname == "log10":
        return torch.log10(a)
    if opname == "cos":
        return torch.cos(a)
    if opname == "sin":
        return torch.sin(a)
    if opname == "tan":
        return torch.tan(a)
    if opname == "erf":
        return torch.erf(a)
    if opname == "gelu":
        return 0.5 * a * (1.0 + torch.erf(a * 0.7071067811865476))
    if opname == "gelu_tanh":
        return 0.5 * a * (1.0 + torch.tanh(0.7978845608028654 * (a + 0.044715 * a * a * a)))
    if opname == "softplus":
        return torch.clamp_min(a, 0) + torch.log1p(torch.exp(-torch.abs(a)))
    if opname == "silu":
        return a * torch.sigmoid(a)
    if opname == "floor":
        return torch.floor(a)
    if opname == "ceil":
        return torch.ceil(a)
    if opname == "sign":
        return torch.sign(a)
    if opname in ("greater", "gt"):
        return (a > b), "pred"
    if opname in ("less", "lt"):
        return (a < b), "pred"
    if opname in ("greater_equal", "ge"):
        return (a >= b), "pred"
    if opname in ("less_equal", "le"):
        return (a <= b), "pred"
    if opname in ("equal", "eq"):
        return (a == b), "pred"
    if opname in ("not_equal", "ne"):
        return (a != b), "pred"          # unordered, as setp.neu (ptxc/expr.py:785-786)
    if opname == "where":
        c = args[0]
        c = c if c.dtype == torch.bool else (c != 0)
        x, y = args[1], args[2]
        if x.dtype != y.dtype:
            y = y.to(x.dtype)
        return torch.where(c, x, y)
    raise OracleError(f"unsupported elementwise op {opname!r}")


def make_inputs(meta: dict, seed_offset: int = 0, rng_kind: str = "normal") -> dict:
    """Seeded inputs exactly as the reference harness builds them.

    ``tools/localrun.py:111-118``: outputs are zeros; ``data`` args are the
    literal values; every other arg is
    ``np.random.default_rng(seed).standard_normal(prod(shape)).astype(dtype)``,
    or, when the argument carries an ``init`` field (benchmark inputs), a
    normal/uniform draw from the same generator.  Returns numpy arrays keyed
    by argument name.
    """
    out = {}
    for a in meta["args"]:
        n = int(np.prod(a["shape"])) if a["shape"] else 1
        dt = NP_DT[a["dtype"]]
        if a.get("output"):
            out[a["name"]] = np.zeros(n, dtype=dt)
        elif "data" in a:
            out[a["name"]] = np.array(a["data"], dtype=dt).reshape(-1)
        else:
            rng = np.random.default_rng(a.get("seed", 0) + seed_offset)
            init = a.get("init")
            if init is None:
                v = rng.standard_normal(n)
            elif init.get("dist") == "normal":
                v = rng.standard_normal(n) * float(init.get("std", 1.0)) + float(init.get("mean", 0.0))
            elif init.get("dist") == "uniform":
                v = rng.uniform(float(init.get("low", 0.0)), float(init.get("high", 1.0)), n)
            else:
                raise OracleError(f"unknown init {init!r}")
            out[a["name"]] = v.astype(dt)
    return out


def run_ir(kernel_op, meta: dict, inputs: dict, blocks=None, threads=None) -> dict:
    """Evaluate the IR on numpy inputs; returns every buffer as numpy (outputs filled)."""
    if threads:
        torch.set_num_threads(threads)
    arrays = {k: np.array(v, copy=True) for k, v in inputs.items()}
    orig = {k: a.dtype for k, a in arrays.items()}
    bufs = {k: torch.from_numpy(a.view(_SIGNED_VIEW[a.dtype]) if a.dtype in _SIGNED_VIEW else a)
            for k, a in arrays.items()}
    with torch.no_grad():
        IRInterpreter(kernel_op, meta, bufs, blocks=blocks).run()
    return {k: v.numpy().view(orig[k]) for k, v in bufs.items()}


def run_chain(pairs, host: dict, blocks=None) -> dict:
    """Evaluate a package of several kernels in order, as the reference harness
    runs them (``tools/localrun.py:160-195``): each kernel's outputs start at
    zero, an ``intermediate`` argument takes the values an earlier kernel wrote
    under that name converted to this argument's dtype, every other input comes
    from ``host``.  ``pairs``: ``[(KernelOp, meta kernel entry), ...]``.
    Returns every output of every kernel by name (the last writer's values)."""
    produced = {}
    for kop, meta in pairs:
        ins = {}
        for a in meta["args"]:
            n = int(np.prod(a["shape"])) if a["shape"] else 1
            dt = NP_DT[a["dtype"]]
            if a.get("output"):
                ins[a["name"]] = np.zeros(n, dtype=dt)
            elif a.get("intermediate"):
                ins[a["name"]] = np.asarray(produced[a["name"]]).reshape(-1).astype(dt)
            else:
                ins[a["name"]] = np.asarray(host[a["name"]]).reshape(-1)
        out = run_ir(kop, meta, ins, blocks=blocks)
        for a in meta["args"]:
            if a.get("output"):
                produced[a["name"]] = out[a["name"]]
    return produced
