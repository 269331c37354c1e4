"""IR synthesiser: Kernel IR + meta.json for the family shapes at any size.

The emmy generator that produced the reference's fixtures is not available,
so the benchmark configurations (which have no fixture) are written here as
IR of the same statement shapes the reference fixtures carry, scaled up:

* row reductions, ``Tile(outer..., aK_co)`` + StridedLoop + WarpShuffle +
  TreeHalve + ``Cond(co == 0)`` write (``tests/variants/v_r_*``, ``w_r_*``);
* rmsnorm / l2norm / softmax: the same plus a second StridedLoop map pass
  (``v_f_rms_512``, ``v_f_l2_256``, ``v_f_softmax_1024``, ``w_f_softmax_dim0``);
* layernorm: a two-moment accumulator pair (sum, sum of squares) and an
  affine map pass (no fixture exists; the formula is the reference spec
  ``tools/specs/ln_specs.py:2-6``);
* f64 matvec: the reduction shape with a second, row-invariant load.

``make_inputs`` builds the seeded inputs as the reference harness does
(``tools/localrun.py:111-118``: ``default_rng(seed).standard_normal``), plus an
optional ``init`` field per argument for the benchmark distributions
(``{"dist": "normal", "mean": m, "std": s}`` or
``{"dist": "uniform", "low": a, "high": b}``, drawn from ``default_rng(seed)``).
"""

from __future__ import annotations

import math

import numpy as np

from .nodes import (
    Accum, Assign, Axis, BinaryExpr, Cond, CpAsyncCommit, CpAsyncCopy, CpAsyncWait, DataType, Dim,
    ElementwiseImpl, Init, KernelOp, Let, Literal, Load, Loop, NpDType, Smem, StridedLoop, Sync,
    Tile, TreeHalve, Var, WarpShuffle, Write,
)

DT = {
    "f32": DataType(name="f32", np=NpDType("float32"), nbytes=4),
    "f16": DataType(name="f16", np=NpDType("float16"), nbytes=2),
    "f64": DataType(name="f64", np=NpDType("float64"), nbytes=8),
}
# integer buffers (the reference's dtype table, ptxc/ops.py:12-25)
INT_NP = {"i8": np.int8, "u8": np.uint8, "i16": np.int16, "u16": np.uint16, "i32": np.int32,
          "u32": np.uint32, "i64": np.int64, "u64": np.uint64}
for _k, _t in INT_NP.items():
    DT[_k] = DataType(name=_k, np=NpDType(np.dtype(_t).name), nbytes=np.dtype(_t).itemsize)
C_NAME = {"f32": "float", "f16": "half", "f64": "double", "i32": "int", "u32": "unsigned",
          "i64": "long", "i16": "short", "i8": "char"}
NP = {"f32": np.float32, "f16": np.float16, "f64": np.float64, **INT_NP}


def V(name):
    return Var(name=name)


def L(v):
    return Literal(value=v, dtype="float" if isinstance(v, float) else "int")


def E(op):
    return ElementwiseImpl(op)


def ax(name, ext):
    return Axis(name=name, extent=Dim(int(ext)), window=None)


def A(name, op, args, dt="f32"):
    return Assign(name=name, op=E(op), args=tuple(args), dtype=DT[dt] if dt else None)


def _combine(states, rule):
    """Combine statements ``state <- rule(state, state__o)`` (sum / max / softmax pair)."""
    if rule == "add":
        return tuple(Assign(name=s, op=E("add"), args=(s, s + "__o"), dtype=None) for s in states)
    if rule == "max":
        return tuple(Assign(name=s, op=E("maximum"), args=(s, s + "__o"), dtype=None) for s in states)
    if rule == "softmax":
        m, s = states
        o = m + "__o"
        return (
            Assign(name=o + "__gn", op=E("maximum"), args=(m, o), dtype=None),
            Assign(name=o + "__dg", op=E("subtract"), args=(m, o + "__gn"), dtype=None),
            Assign(name=o + "__alpha", op=E("exp"), args=(o + "__dg",), dtype=None),
            Assign(name=o + "__dg_o", op=E("subtract"), args=(o, o + "__gn"), dtype=None),
            Assign(name=o + "__beta", op=E("exp"), args=(o + "__dg_o",), dtype=None),
            Assign(name=o + "__" + s + "_sa", op=E("multiply"), args=(o + "__alpha", s), dtype=None),
            Assign(name=o + "__" + s + "_sb", op=E("multiply"), args=(o + "__beta", s + "__o"), dtype=None),
            Assign(name=s, op=E("add"), args=(o + "__" + s + "_sa", o + "__" + s + "_sb"), dtype=None),
            Assign(name=m, op=E("copy"), args=(o + "__gn",), dtype=None),
        )
    raise ValueError(rule)


def _block_combine(states, rule, block, dt="f32"):
    """WarpShuffle + shared slots + TreeHalve, as in every reference reduction fixture."""
    out = [WarpShuffle(state=tuple(states), state_b=tuple(s + "__o" for s in states),
                       combine_states=_combine(states, rule), length=min(32, block), dtype=DT[dt])]
    if block > 32:
        warps = block // 32
        bufs = tuple(s + "_smem" for s in states)
        out += [Smem(name=b, extents=(warps,), dtype=C_NAME[dt], align=0) for b in bufs]
        out.append(Cond(cond=BinaryExpr(op="==", left=V("lane"), right=L(0)),
                        body=tuple(Write(output=b, index=(V("warp"),), values=(s,), value_dtype=DT[dt],
                                         atomic=False, swizzle="NONE") for b, s in zip(bufs, states)),
                        else_body=()))
        out.append(Sync(barrier_id=0, count=None, warp=False))
        out.append(TreeHalve(bufs=bufs, state=tuple(states), state_b=tuple(s + "__o" for s in states),
                             combine_states=_combine(states, rule), length=warps, tid_var="warp",
                             dtype=DT[dt], barrier_id=0, barrier_count=None, inner=None))
    return out


def _arg(name, dtype, shape, **kw):
    d = {"name": name, "dtype": dtype, "shape": [int(s) for s in shape]}
    d.update(kw)
    return d


def _meta(entry, args, grid, block, zero=()):
    return {"node": [a["name"] for a in args if a.get("output")][0], "entry": entry,
            "arg_order": [a["name"] for a in args], "grid": [int(grid), 1, 1],
            "block": [int(block), 1, 1], "smem_bytes": 0, "zero_outputs": list(zero),
            "args": args, "final": True}


def _tile(axes, body, block):
    return Tile(axes=tuple(axes), body=tuple(body), block_threads=int(block), aux_threads=0,
                raster_axes=None, raster_group=None, raster_orient="m")


def _outer_axes(dims):
    return [ax(f"a{i}", d) for i, d in enumerate(dims)]


# ---------------------------------------------------------------------------
# reductions over the last axis


def rmsnorm(rows, cols, eps=1e-5, weight=True, block=128, entry="k_rmsnorm",
            x_init=None, w_init=None):
    """``v_f_rms_512`` shape: ``x * recip(sqrt(eps + sum(x*x)*recip(n))) * w``."""
    co = "a1_co"
    red = StridedLoop(axis=ax("a1", cols), start=V(co), step=L(block), body=(
        Load(names=("in2",), input="x", index=(V("a0"), V("a1")), dtype=DT["f32"]),
        A("v1", "multiply", ("in2", "in2")),
        Accum(name="acc0", value="v1", op=E("add"), dtype=DT["f32"], axes=("a1",), base=None),
    ), unroll=False, end=None, seed=True)
    mp = [Load(names=("in3",), input="x", index=(V("a0"), V("a2")), dtype=DT["f32"]),
          A("v6", "multiply", ("in3", "v5"))]
    if weight:
        mp += [Load(names=("in4",), input="w", index=(V("a2"),), dtype=DT["f32"]),
               A("v7", "multiply", ("in4", "v6"))]
    mp.append(Write(output="y", index=(V("a0"), V("a2")), values=("v7" if weight else "v6",),
                    value_dtype=DT["f32"], atomic=False, swizzle="NONE"))
    body = [red] + _block_combine(["acc0"], "add", block) + [
        Load(names=("in1",), input="mean_count", index=(L(0),), dtype=DT["f32"]),
        A("v0", "reciprocal", ("in1",)),
        A("v2", "multiply", ("acc0", "v0")),
        Load(names=("in0",), input="add_c1", index=(L(0),), dtype=DT["f32"]),
        A("v3", "add", ("in0", "v2")),
        A("v4", "sqrt", ("v3",)),
        A("v5", "reciprocal", ("v4",)),
        StridedLoop(axis=ax("a2", cols), start=V(co), step=L(block), body=tuple(mp),
                    unroll=False, end=None, seed=True),
    ]
    kop = KernelOp(name=entry, body=(_tile([ax("a0", rows), ax(co, block)], body, block),))
    args = [_arg("mean_count", "f32", [1], data=[float(cols)]),
            _arg("add_c1", "f32", [1], data=[float(eps)]),
            _arg("x", "f32", [rows, cols], seed=0, **({"init": x_init} if x_init else {}))]
    if weight:
        args.append(_arg("w", "f32", [cols], seed=1, **({"init": w_init} if w_init else {})))
    args.append(_arg("y", "f32", [rows, cols], output=True))
    return kop, _meta(entry, args, rows, block)


def l2norm(rows, cols, block=128, entry="k_l2norm"):
    """``v_f_l2_256`` shape: ``x * recip(sqrt(sum(x*x)))``."""
    co = "a1_co"
    body = [StridedLoop(axis=ax("a1", cols), start=V(co), step=L(block), body=(
        Load(names=("in0",), input="x", index=(V("a0"), V("a1")), dtype=DT["f32"]),
        A("v0", "multiply", ("in0", "in0")),
        Accum(name="acc0", value="v0", op=E("add"), dtype=DT["f32"], axes=("a1",), base=None),
    ), unroll=False, end=None, seed=True)] + _block_combine(["acc0"], "add", block) + [
        A("v1", "sqrt", ("acc0",)), A("v2", "reciprocal", ("v1",)),
        StridedLoop(axis=ax("a2", cols), start=V(co), step=L(block), body=(
            Load(names=("in1",), input="x", index=(V("a0"), V("a2")), dtype=DT["f32"]),
            A("v3", "multiply", ("in1", "v2")),
            Write(output="y", index=(V("a0"), V("a2")), values=("v3",), value_dtype=DT["f32"],
                  atomic=False, swizzle="NONE"),
        ), unroll=False, end=None, seed=True)]
    kop = KernelOp(name=entry, body=(_tile([ax("a0", rows), ax(co, block)], body, block),))
    args = [_arg("x", "f32", [rows, cols], seed=0), _arg("y", "f32", [rows, cols], output=True)]
    return kop, _meta(entry, args, rows, block)


def _softmax_update(x, m, s, one="one"):
    return (
        Assign(name=x + "__gn", op=E("maximum"), args=(m, x), dtype=DT["f32"]),
        Assign(name=x + "__dg", op=E("subtract"), args=(m, x + "__gn"), dtype=DT["f32"]),
        Assign(name=x + "__alpha", op=E("exp"), args=(x + "__dg",), dtype=DT["f32"]),
        Assign(name=x + "__dg_o", op=E("subtract"), args=(x, x + "__gn"), dtype=DT["f32"]),
        Assign(name=x + "__beta", op=E("exp"), args=(x + "__dg_o",), dtype=DT["f32"]),
        Assign(name=x + "__" + s + "_sa", op=E("multiply"), args=(s, x + "__alpha"), dtype=DT["f32"]),
        Assign(name=x + "__" + s + "_sb", op=E("multiply"), args=(x + "__beta", one), dtype=DT["f32"]),
    )


def softmax(shape, dim=-1, block=128, entry="k_softmax", x_init=None):
    """``v_f_softmax_1024`` (last axis, any rank) or ``w_f_softmax_dim0`` (2-D, dim 0) shape."""
    shape = [int(s) for s in shape]
    nd = len(shape)
    dim = dim % nd
    if dim == nd - 1:
        outer = shape[:-1]
        n = shape[-1]
        k = len(outer)
        co = f"a{k}_co"
        r, m = f"a{k}", f"a{k + 1}"
        idx_r = tuple(V(f"a{i}") for i in range(k)) + (V(r),)
        idx_m = tuple(V(f"a{i}") for i in range(k)) + (V(m),)
        axes = _outer_axes(outer) + [ax(co, block)]
        grid = math.prod(outer) if outer else 1
    elif nd == 2 and dim == 0:
        n, cols = shape
        co = "a2_co"
        r = "a2"
        idx_r = (V("a2"), V("a1"))
        axes = [ax("a0", n), ax("a1", cols), ax(co, block)]
        grid = n * cols
    else:
        raise ValueError("softmax synthesis covers the last axis, or dim 0 of a 2-D tensor")
    red = StridedLoop(axis=ax(r, n), start=V(co), step=L(block), body=(
        Let(name="one", value=L(1.0), dtype=DT["f32"]),
        Load(names=("in0",), input="x", index=idx_r, dtype=DT["f32"]),
    ) + _softmax_update("in0", "acc0", "acc1") + (
        Accum(name="acc1", value="in0__acc1_sb", op=E("add"), dtype=DT["f32"], axes=(r,),
              base="in0__acc1_sa"),
        Accum(name="acc0", value="in0", op=E("maximum"), dtype=DT["f32"], axes=(r,), base=None),
    ), unroll=False, end=None, seed=True)
    tail_ops = [A("v3", "subtract", ("in2", "acc0")), A("v4", "exp", ("v3",)),
                A("v5", "multiply", ("v2", "v4"))]
    if dim == nd - 1:
        out = [A("v2", "reciprocal", ("acc1",)),
               StridedLoop(axis=ax(m, n), start=V(co), step=L(block), body=tuple(
                   [Load(names=("in2",), input="x", index=idx_m, dtype=DT["f32"])] + tail_ops + [
                       Write(output="y", index=idx_m, values=("v5",), value_dtype=DT["f32"],
                             atomic=False, swizzle="NONE")]), unroll=False, end=None, seed=True)]
    else:
        out = [Cond(cond=BinaryExpr(op="==", left=V(co), right=L(0)), body=tuple(
            [A("v2", "reciprocal", ("acc1",)),
             Load(names=("in2",), input="x", index=(V("a0"), V("a1")), dtype=DT["f32"])] + tail_ops + [
                Write(output="y", index=(V("a0"), V("a1")), values=("v5",), value_dtype=DT["f32"],
                      atomic=False, swizzle="NONE")]), else_body=())]
    body = [red] + _block_combine(["acc0", "acc1"], "softmax", block) + out
    kop = KernelOp(name=entry, body=(_tile(axes, body, block),))
    args = [_arg("x", "f32", shape, seed=0, **({"init": x_init} if x_init else {})),
            _arg("y", "f32", shape, output=True)]
    return kop, _meta(entry, args, grid, block)


def layernorm(rows, cols, eps=1e-5, affine=True, block=128, entry="k_layernorm",
              x_init=None, g_init=None, b_init=None):
    """Two-moment layernorm: ``(x - mean) * recip(sqrt(E[x^2] - mean^2 + eps)) * g + b``."""
    co = "a1_co"
    red = StridedLoop(axis=ax("a1", cols), start=V(co), step=L(block), body=(
        Load(names=("in0",), input="x", index=(V("a0"), V("a1")), dtype=DT["f32"]),
        A("v0", "multiply", ("in0", "in0")),
        Accum(name="acc0", value="in0", op=E("add"), dtype=DT["f32"], axes=("a1",), base=None),
        Accum(name="acc1", value="v0", op=E("add"), dtype=DT["f32"], axes=("a1",), base=None),
    ), unroll=False, end=None, seed=True)
    mp = [Load(names=("in3",), input="x", index=(V("a0"), V("a2")), dtype=DT["f32"]),
          A("v9", "subtract", ("in3", "v2")), A("v10", "multiply", ("v9", "v8"))]
    last = "v10"
    if affine:
        mp += [Load(names=("in4",), input="gamma", index=(V("a2"),), dtype=DT["f32"]),
               A("v11", "multiply", ("v10", "in4")),
               Load(names=("in5",), input="beta", index=(V("a2"),), dtype=DT["f32"]),
               A("v12", "add", ("v11", "in5"))]
        last = "v12"
    mp.append(Write(output="y", index=(V("a0"), V("a2")), values=(last,), value_dtype=DT["f32"],
                    atomic=False, swizzle="NONE"))
    body = [red] + _block_combine(["acc0", "acc1"], "add", block) + [
        Load(names=("in1",), input="ln_count", index=(L(0),), dtype=DT["f32"]),
        A("v1", "reciprocal", ("in1",)),
        A("v2", "multiply", ("acc0", "v1")),
        A("v3", "multiply", ("acc1", "v1")),
        A("v4", "multiply", ("v2", "v2")),
        A("v5", "subtract", ("v3", "v4")),
        Load(names=("in2",), input="ln_eps", index=(L(0),), dtype=DT["f32"]),
        A("v6", "add", ("v5", "in2")),
        A("v7", "sqrt", ("v6",)),
        A("v8", "reciprocal", ("v7",)),
        StridedLoop(axis=ax("a2", cols), start=V(co), step=L(block), body=tuple(mp),
                    unroll=False, end=None, seed=True),
    ]
    kop = KernelOp(name=entry, body=(_tile([ax("a0", rows), ax(co, block)], body, block),))
    args = [_arg("ln_count", "f32", [1], data=[float(cols)]),
            _arg("ln_eps", "f32", [1], data=[float(eps)]),
            _arg("x", "f32", [rows, cols], seed=0, **({"init": x_init} if x_init else {}))]
    if affine:
        args.append(_arg("gamma", "f32", [cols], seed=1, **({"init": g_init} if g_init else {})))
        args.append(_arg("beta", "f32", [cols], seed=2, **({"init": b_init} if b_init else {})))
    args.append(_arg("y", "f32", [rows, cols], output=True))
    return kop, _meta(entry, args, rows, block)


def reduce(shape, axis=-1, op="sum", block=128, entry="k_reduce", dtype="f32"):
    """Sum / mean / max over one axis (``v_r_*``, ``w_r_dim0``, ``w_r_mid`` shapes).

    ``axis=None`` reduces a 1-D tensor to a scalar (``v_r_100000``).
    """
    shape = [int(s) for s in shape]
    if axis is None:
        assert len(shape) == 1
        kept, n = [], shape[0]
        co, r = "a0_co", "a0"
        idx = (V(r),)
    else:
        axis = axis % len(shape)
        kept = [d for i, d in enumerate(shape) if i != axis]
        n = shape[axis]
        k = len(kept)
        co, r = f"a{k}_co", f"a{k}"
        coords = [V(f"a{i}") for i in range(k)]
        idx = tuple(coords[:axis]) + (V(r),) + tuple(coords[axis:])
    fold = {"sum": "add", "mean": "add", "max": "maximum", "min": "minimum"}[op]
    red = StridedLoop(axis=ax(r, n), start=V(co), step=L(block), body=(
        Load(names=("in0",), input="x", index=idx, dtype=DT[dtype]),
        Accum(name="acc0", value="in0", op=E(fold), dtype=DT[dtype], axes=(r,), base=None),
    ), unroll=False, end=None, seed=True)
    out_idx = tuple(V(f"a{i}") for i in range(len(kept)))
    wbody = []
    args = []
    val = "acc0"
    if op == "mean":
        wbody = [Load(names=("in1",), input="mean_count", index=(L(0),), dtype=DT[dtype]),
                 A("v0", "reciprocal", ("in1",), dtype), A("v1", "multiply", ("acc0", "v0"), dtype)]
        val = "v1"
        args.append(_arg("mean_count", dtype, [1], data=[float(n)]))
    wbody.append(Write(output="y", index=out_idx, values=(val,), value_dtype=DT[dtype],
                       atomic=False, swizzle="NONE"))
    rule = "max" if fold == "maximum" else ("add" if fold == "add" else None)
    if rule is None:
        raise ValueError("min reductions have no synthesised combine")
    body = [red] + _block_combine(["acc0"], rule, block, dtype) + [
        Cond(cond=BinaryExpr(op="==", left=V(co), right=L(0)), body=tuple(wbody), else_body=())]
    axes = _outer_axes(kept) + [ax(co, block)]
    kop = KernelOp(name=entry, body=(_tile(axes, body, block),))
    args += [_arg("x", dtype, shape, seed=0), _arg("y", dtype, kept if kept else [1], output=True)]
    return kop, _meta(entry, args, math.prod(kept) if kept else 1, block)


def matvec(rows, cols, dtype="f64", block=128, entry="k_matvec"):
    """``y = A @ v``: the reduction shape with a row-invariant second load."""
    co = "a1_co"
    red = StridedLoop(axis=ax("a1", cols), start=V(co), step=L(block), body=(
        Load(names=("in0",), input="A", index=(V("a0"), V("a1")), dtype=DT[dtype]),
        Load(names=("in1",), input="v", index=(V("a1"),), dtype=DT[dtype]),
        A("v0", "multiply", ("in0", "in1"), dtype),
        Accum(name="acc0", value="v0", op=E("add"), dtype=DT[dtype], axes=("a1",), base=None),
    ), unroll=False, end=None, seed=True)
    body = [red] + _block_combine(["acc0"], "add", block, dtype) + [
        Cond(cond=BinaryExpr(op="==", left=V(co), right=L(0)), body=(
            Write(output="y", index=(V("a0"),), values=("acc0",), value_dtype=DT[dtype],
                  atomic=False, swizzle="NONE"),), else_body=())]
    kop = KernelOp(name=entry, body=(_tile([ax("a0", rows), ax(co, block)], body, block),))
    args = [_arg("A", dtype, [rows, cols], seed=0), _arg("v", dtype, [cols], seed=1),
            _arg("y", dtype, [rows], output=True)]
    return kop, _meta(entry, args, rows, block)


# ---------------------------------------------------------------------------
# inputs


def make_inputs(meta: dict, seed_offset: int = 0, only=None) -> dict:
    """Seeded host inputs (numpy) for every argument, outputs zero-filled.

    Integer arguments draw uniformly from the dtype's range (or from
    ``{"dist": "int", "low": a, "high": b}``); a float ``init`` on an integer
    argument is drawn as floats and truncated toward zero."""
    out = {}
    for a in meta["args"]:
        if only is not None and a["name"] not in only:
            continue
        n = math.prod(a["shape"]) if a["shape"] else 1
        dt = NP.get(a["dtype"], np.float32)
        if a.get("output"):
            out[a["name"]] = np.zeros(n, dtype=dt)
        elif "data" in a:
            out[a["name"]] = np.array(a["data"], dtype=dt).reshape(-1)
        else:
            rng = np.random.default_rng(a.get("seed", 0) + seed_offset)
            init = a.get("init")
            if np.dtype(dt).kind in "iu" and (init is None or init.get("dist") == "int"):
                # integers: the dtype's whole range, or {"dist": "int", "low", "high"}
                # (both ends included)
                info = np.iinfo(dt)
                lo = info.min if init is None else max(int(init["low"]), int(info.min))
                hi = info.max if init is None else min(int(init["high"]), int(info.max))
                out[a["name"]] = rng.integers(lo, hi, size=n, endpoint=True, dtype=dt)
                continue
            if init is None:
                v = rng.standard_normal(n)
            elif init.get("dist") == "normal":
                v = rng.standard_normal(n) * float(init.get("std", 1.0)) + float(init.get("mean", 0.0))
            elif init.get("dist") == "uniform":
                v = rng.uniform(float(init.get("low", 0.0)), float(init.get("high", 1.0)), n)
            else:
                raise ValueError(f"unknown init {init!r}")
            out[a["name"]] = v.astype(dt)
    return out


# ---------------------------------------------------------------------------
# tiled matmul (w_m_batch / v_m_rect_small shape)


def _B(op, left, right):
    return BinaryExpr(op=op, left=left, right=right)


def matmul(M, N, K, batch=1, splits=1, dtype="f32", out_dtype=None, bias=False, relu=False,
           tm=64, tn=64, rm=4, rn=4, bk=None, entry="k_matmul", a_init=None, b_init=None,
           bias_init=None, c_name="C"):
    """``C = A @ B`` (+ bias, relu) in the reference's cp.async tiled-matmul shape.

    Tile axes ``(_aS_ks?, a0? (batch), a1_b, a2_b, a1_u, a2_u)``: per split and
    batch, a (tm x tn) output block computed by (tm/rm) x (tn/rn) threads, each
    holding an rm x rn accumulator micro-tile (``Init`` seeds); per K step
    ``bk`` the block stages A[tm, bk] and B[bk, tn] through ``CpAsyncCopy`` of
    16 bytes into ``_a_smem`` / ``_b_smem``, then an unrolled ``Loop _ki``
    folds smem products into the accumulators; writes are atomic when K is
    split (``zero_outputs`` names C), as in ``tests/variants/w_m_batch``.
    """
    out_dtype = out_dtype or dtype
    bias_dt = "f64" if dtype == "f64" else "f32"
    esz = {"f32": 4, "f16": 2, "f64": 8}[dtype]
    vec = 16 // esz                                # elements per 16-byte copy
    bk = bk or (16 if dtype == "f32" else 32)
    assert M % tm == 0 and N % tn == 0 and tm % rm == 0 and tn % rn == 0
    assert K % splits == 0 and (K // splits) % bk == 0 and bk % vec == 0 and tn % vec == 0
    ksplit = K // splits
    mu, nu = tm // rm, tn // rn
    threads = mu * nu
    axes = []
    if splits > 1:
        axes.append(ax("_a3_ks", splits))
    if batch > 1:
        axes.append(ax("a0", batch))
    axes += [Axis(name="a1_b", extent=Dim(M // tm), window=None),
             Axis(name="a2_b", extent=Dim(N // tn), window=None),
             ax("a1_u", mu), ax("a2_u", nu)]
    tid = _B("+", _B("*", V("a1_u"), L(nu)), V("a2_u"))
    kbase = _B("*", V("_a3_ks"), L(ksplit)) if splits > 1 else L(0)
    bidx = (V("a0"),) if batch > 1 else ()
    body = []
    for i in range(rm):
        for j in range(rn):
            body.append(Init(name=f"acc0__c{i}_{j}", identity=0.0, dtype=DT["f32"]))
    body += [Smem(name="_a_smem", extents=(tm, bk), dtype=C_NAME[dtype], align=16),
             Smem(name="_b_smem", extents=(bk, tn), dtype=C_NAME[dtype], align=16)]
    a_chunks = tm * bk // vec
    b_chunks = bk * tn // vec
    fa = _B("*", V("_fa"), L(vec))
    fb = _B("*", V("_fb"), L(vec))
    copy_a = StridedLoop(axis=ax("_fa", a_chunks), start=tid, step=L(threads), body=(
        CpAsyncCopy(
            smem="_a_smem", smem_index=(_B("/", fa, L(bk)), _B("%", fa, L(bk))), src="A",
            src_index=bidx + (_B("+", _B("*", V("a1_b"), L(tm)), _B("/", fa, L(bk))),
                              _B("+", kbase, _B("+", V("_ks"), _B("%", fa, L(bk))))),
            nbytes=16, swizzle="NONE", lane_index=None, lane_rows=0),), unroll=False, end=None, seed=True)
    copy_b = StridedLoop(axis=ax("_fb", b_chunks), start=tid, step=L(threads), body=(
        CpAsyncCopy(
            smem="_b_smem", smem_index=(_B("/", fb, L(tn)), _B("%", fb, L(tn))), src="B",
            src_index=bidx + (_B("+", kbase, _B("+", V("_ks"), _B("/", fb, L(tn)))),
                              _B("+", _B("*", V("a2_b"), L(tn)), _B("%", fb, L(tn)))),
            nbytes=16, swizzle="NONE", lane_index=None, lane_rows=0),), unroll=False, end=None, seed=True)
    inner = []
    for i in range(rm):
        row_l = _B("-", _B("+", _B("+", _B("*", V("a1_b"), L(tm)), _B("*", V("a1_u"), L(rm))), L(i)),
                   _B("*", V("a1_b"), L(tm)))
        inner.append(Load(names=(f"in0__c{i}_0",), input="_a_smem", index=(row_l, V("_ki")), dtype=None))
        for j in range(rn):
            if i == 0:
                col_l = _B("-", _B("+", _B("+", _B("*", V("a2_b"), L(tn)), _B("*", V("a2_u"), L(rn))), L(j)),
                           _B("*", V("a2_b"), L(tn)))
                inner.append(Load(names=(f"in1__c0_{j}",), input="_b_smem", index=(V("_ki"), col_l), dtype=None))
            inner.append(A(f"acc0__v__c{i}_{j}", "multiply", (f"in1__c0_{j}", f"in0__c{i}_0")))
            inner.append(Accum(name=f"acc0__c{i}_{j}", value=f"acc0__v__c{i}_{j}", op=E("add"),
                               dtype=DT["f32"], axes=("_ki",), base=None))
    body.append(StridedLoop(axis=ax("_ks", ksplit), start=L(0), step=L(bk), body=(
        copy_a, copy_b, CpAsyncCommit(), CpAsyncWait(group=0), Sync(barrier_id=0, count=None, warp=False),
        Loop(axis=ax("_ki", bk), body=tuple(inner), unroll=True, seed=False),
        Sync(barrier_id=0, count=None, warp=False)), unroll=False, end=None, seed=True))
    for i in range(rm):
        row = _B("+", _B("+", _B("*", V("a1_b"), L(tm)), _B("*", V("a1_u"), L(rm))), L(i))
        for j in range(rn):
            col = _B("+", _B("+", _B("*", V("a2_b"), L(tn)), _B("*", V("a2_u"), L(rn))), L(j))
            val = f"acc0__c{i}_{j}"
            if bias:
                body.append(Load(names=(f"bias__c{i}_{j}",), input="bias", index=(col,), dtype=DT[bias_dt]))
                body.append(A(f"v0__c{i}_{j}", "add", (val, f"bias__c{i}_{j}")))
                val = f"v0__c{i}_{j}"
            if relu:
                body.append(Let(name=f"zero__c{i}_{j}", value=L(0.0), dtype=DT["f32"]))
                body.append(A(f"v1__c{i}_{j}", "maximum", (val, f"zero__c{i}_{j}")))
                val = f"v1__c{i}_{j}"
            body.append(Write(output=c_name, index=bidx + (row, col), values=(val,), value_dtype=DT[out_dtype],
                              atomic=splits > 1, swizzle="NONE"))
    tile = Tile(axes=tuple(axes), body=tuple(body), block_threads=threads, aux_threads=0,
                raster_axes=("a1_b", "a2_b"), raster_group=None, raster_orient="m")
    kop = KernelOp(name=entry, body=(tile,))
    lead = [batch] if batch > 1 else []
    args = [_arg("B", dtype, lead + [K, N], seed=1, **({"init": b_init} if b_init else {})),
            _arg("A", dtype, lead + [M, K], seed=0, **({"init": a_init} if a_init else {}))]
    if bias:
        args.append(_arg("bias", bias_dt, [N], seed=2, **({"init": bias_init} if bias_init else {})))
    args.append(_arg(c_name, out_dtype, lead + [M, N], output=True))
    nblocks = splits * batch * (M // tm) * (N // tn)
    return kop, _meta(entry, args, nblocks, threads, zero=[c_name] if splits > 1 else [])


# ---------------------------------------------------------------------------
# attention-like chain (w_a_head64 shape, with batch and head Tile axes)


def attention(B, H, S, D, dtype="f16", out_dtype=None, scale_div=None, entry="k_attention",
              q_init=None, k_init=None, v_init=None, k_transposed=False, Dv=None):
    """``softmax(q @ k^T * recip(div)) @ v`` per (batch, head), in the shape of
    ``tests/variants/w_a_head64``: one thread per output element (query row,
    value column) walks the keys in a ``Loop``, each key's score is an inner
    ``Loop`` dot product over the head dim, followed by the online max/sum
    update and the rescaled accumulation of ``v``; the write divides by the
    sum.  ``q, k, v, out`` are ``[B, H, S, D]`` (k not pre-transposed).
    """
    out_dtype = out_dtype or dtype
    Dv = Dv or D
    div = float(scale_div if scale_div is not None else math.sqrt(D))
    rows_u, cols_u = 1, max(c for c in range(1, min(Dv, 64) + 1) if Dv % c == 0)
    threads = rows_u * cols_u
    axes = [ax("a6", B), ax("a7", H),
            Axis(name="a0_b", extent=Dim(S // rows_u), window=None),
            Axis(name="a5_b", extent=Dim(Dv // cols_u), window=None),
            ax("a0_u", rows_u), ax("a5_u", cols_u)]
    row = _B("+", _B("+", _B("*", V("a0_b"), L(rows_u)), _B("*", V("a0_u"), L(1))), L(0))
    col = _B("+", _B("+", _B("*", V("a5_b"), L(cols_u)), _B("*", V("a5_u"), L(1))), L(0))
    bh = (V("a6"), V("a7"))
    f = "f32"
    dot = Loop(axis=ax("a2", D), body=(
        Load(names=("in2__ar0",), input="q", index=bh + (row, V("a2")), dtype=DT[dtype]),
        Load(names=("in1__ar0",), input="k",
             index=bh + ((V("a2"), V("a1")) if k_transposed else (V("a1"), V("a2"))), dtype=DT[dtype]),
        A("v3__ar0", "multiply", ("in1__ar0", "in2__ar0")),
        Accum(name="acc0__ar0", value="v3__ar0", op=E("add"), dtype=DT[f], axes=("a2",), base=None),
    ), unroll=False, seed=True)
    x = "v4__c0_0"
    keys = Loop(axis=ax("a1", S), body=(
        dot,
        A(x, "multiply", ("acc0__ar0", "v1")),
        Let(name="one__c0_0", value=L(1.0), dtype=DT[f]),
        A(x + "__gn", "maximum", ("acc1__c0_0", x)),
        A(x + "__dg", "subtract", ("acc1__c0_0", x + "__gn")),
        A(x + "__alpha", "exp", (x + "__dg",)),
        A(x + "__dg_o", "subtract", (x, x + "__gn")),
        A(x + "__beta", "exp", (x + "__dg_o",)),
        A(x + "__acc3_sa", "multiply", ("acc3__c0_0", x + "__alpha")),
        A(x + "__acc3_sb", "multiply", ("one__c0_0", x + "__beta")),
        Accum(name="acc3__c0_0", value=x + "__acc3_sb", op=E("add"), dtype=DT[f], axes=("a1",),
              base=x + "__acc3_sa"),
        A(x + "__acc5__sum_sa", "multiply", ("acc5__sum__c0_0", x + "__alpha")),
        Load(names=("in7__bc0",), input="v", index=bh + (V("a1"), col), dtype=DT[dtype]),
        A(x + "__acc5__sum_sb", "multiply", ("in7__bc0", x + "__beta")),
        Accum(name="acc5__sum__c0_0", value=x + "__acc5__sum_sb", op=E("add"), dtype=DT[f],
              axes=("a1",), base=x + "__acc5__sum_sa"),
        Accum(name="acc1__c0_0", value=x, op=E("maximum"), dtype=DT[f], axes=("a1",), base=None),
    ), unroll=False, seed=True)
    body = [
        Load(names=("in0",), input="div_c1", index=(L(0),), dtype=DT[f]),
        A("v1", "reciprocal", ("in0",)),
        keys,
        A("v9__c0_0", "reciprocal", ("acc3__c0_0",)),
        A("acc5__c0_0", "multiply", ("acc5__sum__c0_0", "v9__c0_0")),
        Write(output="o", index=bh + (row, col), values=("acc5__c0_0",), value_dtype=DT[out_dtype],
              atomic=False, swizzle="NONE"),
    ]
    tile = Tile(axes=tuple(axes), body=tuple(body), block_threads=threads, aux_threads=0,
                raster_axes=("a0_b", "a5_b"), raster_group=None, raster_orient="m")
    kop = KernelOp(name=entry, body=(tile,))
    shp = [B, H, S, D]
    args = [_arg("div_c1", "f32", [1], data=[div]),
            _arg("q", dtype, shp, seed=0, **({"init": q_init} if q_init else {})),
            _arg("k", dtype, [B, H, D, S] if k_transposed else shp, seed=1,
                 **({"init": k_init} if k_init else {})),
            _arg("v", dtype, [B, H, S, Dv], seed=2, **({"init": v_init} if v_init else {})),
            _arg("o", out_dtype, [B, H, S, Dv], output=True)]
    return kop, _meta(entry, args, B * H * S * Dv // threads, threads)


# ---------------------------------------------------------------------------
# pointwise (v_p_* / w_p_* shape)

BOOL = DataType(name="bool", np=NpDType("bool"), nbytes=1)
_COMPARE = {"greater", "less", "greater_equal", "less_equal", "equal", "not_equal"}
# predicate-valued ops of the reference's Assign (ptxc/stmts.py:516-518, ptxc/common.py:20-23)
_LOGICAL = {"logical_and", "logical_or", "logical_not", "bitwise_and", "bitwise_or",
            "bitwise_not", "and", "or", "not"}


def pointwise(n, expr, dtype="f32", shape=None, block=256, unroll=None, entry="k_pointwise",
              vector_write=True, inits=None, out="out", seeds=None, tile_shape=None, dtypes=None,
              out_dtype=None):
    """The reference pointwise shape: ``Tile(a0 : n/U)`` with U unrolled copies.

    Each copy u loads its element ``a0*U + u`` of every input, loads the
    one-element constant tensors at index 0, evaluates ``expr`` with one Assign
    per op (typed ``dtype``; comparisons typed bool) and the copies' results
    are written by one vector Write (``vector_write``) or U scalar Writes --
    ``v_p_big`` / ``w_p_f64`` respectively.  ``expr`` is a nested tuple:
    ``"x0"`` names an input tensor of ``shape`` (default ``[n]``),
    ``("const", name, value)`` a one-element constant tensor, ``("imm", value)``
    an immediate (Let), and ``(op, arg, ...)`` an elementwise op.  Broadcast
    inputs: ``("bcast", name, numel, D, M)`` reads ``name[(e // D) % M]`` for
    element e (``M = 0``: no ``%``); with ``tile_shape`` (a multi-axis Tile,
    one element per thread, axes ``a0, a1, ...``), ``("axis", name, (i, ...))``
    reads ``name[a_i, ...]``.  Inputs get seeds 0, 1, ... in order of first
    use unless ``seeds`` names them; ``dtypes`` overrides an input's dtype and
    ``out_dtype`` the output's (Assigns stay ``dtype``).
    """
    shape = list(shape) if shape else [int(n)]
    if math.prod(shape) != n:
        raise ValueError("shape does not hold n elements")
    if tile_shape is not None:
        if math.prod(tile_shape) != n:
            raise ValueError("tile_shape does not hold n elements")
        unroll = 1
    if unroll is None:
        unroll = next(u for u in (4, 3, 2, 1) if n % u == 0)
    if n % unroll:
        raise ValueError("unroll must divide n")
    T = n // unroll
    inputs, consts, bshapes = [], {}, {}

    def walk(e):
        if isinstance(e, str):
            if e not in inputs:
                inputs.append(e)
        elif e[0] == "const":
            consts[e[1]] = int(e[2]) if dtype in INT_NP else float(e[2])
        elif e[0] == "bcast":
            if e[1] not in inputs:
                inputs.append(e[1])
            bshapes[e[1]] = [int(e[2])]
        elif e[0] == "axis":
            if e[1] not in inputs:
                inputs.append(e[1])
            bshapes[e[1]] = [int(tile_shape[i]) for i in e[2]]
        elif e[0] != "imm":
            for a in e[1:]:
                walk(a)
    walk(expr)

    def lin_of(u):
        if tile_shape is not None:
            lin = V("a0")
            for i in range(1, len(tile_shape)):
                lin = _B("+", _B("*", lin, L(int(tile_shape[i]))), V(f"a{i}"))
            return lin
        return _B("+", _B("*", V("a0"), L(unroll)), L(u)) if T > 1 else L(u)

    def flat_index(u):
        if tile_shape is not None and list(tile_shape) == list(shape):
            return tuple(V(f"a{i}") for i in range(len(shape)))
        lin = lin_of(u)
        if len(shape) == 1:
            return (lin,)
        idx = []
        for i in range(len(shape)):
            stride = math.prod(shape[i + 1:])
            c = _B("//", lin, L(stride)) if i < len(shape) - 1 else lin
            idx.append(_B("%", c, L(shape[i])) if i > 0 else c)
        return tuple(idx)

    body = []
    results = []
    for u in range(unroll):
        counter = [0]
        loaded = {}

        def in_dt(name):
            return DT[dtypes[name]] if dtypes and name in dtypes else DT[dtype]

        def emit(e):
            if isinstance(e, str):
                if e not in loaded:
                    nm = f"in{inputs.index(e)}__u{u}"
                    body.append(Load(names=(nm,), input=e, index=flat_index(u), dtype=in_dt(e)))
                    loaded[e] = nm
                return loaded[e]
            if e[0] in ("bcast", "axis"):
                key = (e[0], e[1])
                if key not in loaded:
                    nm = f"in{inputs.index(e[1])}b__u{u}"
                    if e[0] == "axis":
                        idx = tuple(V(f"a{i}") for i in e[2])
                    else:
                        q = _B("//", lin_of(u), L(int(e[3]))) if int(e[3]) > 1 else lin_of(u)
                        idx = (_B("%", q, L(int(e[4]))) if int(e[4]) else q,)
                    body.append(Load(names=(nm,), input=e[1], index=idx, dtype=in_dt(e[1])))
                    loaded[key] = nm
                return loaded[key]
            if e[0] == "const":
                nm = f"c_{e[1]}__u{u}"
                if nm not in loaded:
                    body.append(Load(names=(nm,), input=e[1], index=(L(0),), dtype=DT[dtype]))
                    loaded[nm] = nm
                return nm
            if e[0] == "imm":
                nm = f"k{counter[0]}__u{u}"
                counter[0] += 1
                body.append(Let(name=nm, value=L(int(e[1]) if dtype in INT_NP else float(e[1])),
                                dtype=DT[dtype]))
                return nm
            args = [emit(a) for a in e[1:]]
            nm = f"v{counter[0]}__u{u}"
            counter[0] += 1
            dt = BOOL if e[0] in _COMPARE or e[0] in _LOGICAL else DT[dtype]
            body.append(Assign(name=nm, op=E(e[0]), args=tuple(args), dtype=dt))
            return nm
        results.append(emit(expr))
    base = _B("*", V("a0"), L(unroll)) if T > 1 else L(0)
    odt = DT[out_dtype or dtype]
    if tile_shape is not None:
        body.append(Write(output=out, index=flat_index(0), values=(results[0],), value_dtype=odt,
                          atomic=False, swizzle="NONE"))
    elif vector_write:
        body.append(Write(output=out, index=(_B("+", base, L(0)) if T > 1 else L(0),),
                          values=tuple(results), value_dtype=odt, atomic=False,
                          swizzle="NONE"))
    else:
        for u, r in enumerate(results):
            body.append(Write(output=out, index=(_B("+", base, L(u)) if T > 1 else L(u),),
                              values=(r,), value_dtype=odt, atomic=False, swizzle="NONE"))
    axes = ([ax(f"a{i}", int(e)) for i, e in enumerate(tile_shape)] if tile_shape is not None
            else [ax("a0", T)])
    kop = KernelOp(name=entry, body=(_tile(axes, body, block),))
    args = [_arg(c, dtype, [1], data=[v]) for c, v in consts.items()]
    for i, name in enumerate(inputs):
        kw = {"init": inits[name]} if inits and name in inits else {}
        seed = seeds[name] if seeds and name in seeds else i
        dt = dtypes[name] if dtypes and name in dtypes else dtype
        args.append(_arg(name, dt, bshapes.get(name, shape), seed=seed, **kw))
    args.append(_arg(out, out_dtype or dtype, shape, output=True))
    return kop, _meta(entry, args, (T + block - 1) // block, block)


def mm_bias_relu_chain(M, N, K, dtype="f32", c_dtype=None, out_dtype=None, compute=None,
                       bias=True, relu=True, batch=1, axis_form=True, **mm_kw):
    """The two-kernel matmul + bias + ReLU package (the reference's
    ``adv_mm_bias_relu``: ``k_relu__partial`` -> ``k_relu``).

    Kernel 1 (``final: false``) writes the product ``mm`` (dtype ``c_dtype``);
    kernel 2 reads it as an intermediate and writes
    ``out = relu(mm + bias[n])`` (``out_dtype``), its Assigns typed
    ``compute`` (default f32).  ``axis_form``: kernel 2 is a two-axis Tile
    reading ``bias[a1]``; else a flat Tile reading ``bias[e % N]``.
    Returns ``[(KernelOp, meta kernel entry), ...]``.
    """
    c_dtype = c_dtype or dtype
    out_dtype = out_dtype or c_dtype
    compute = compute or "f32"
    k1, m1 = matmul(M, N, K, batch=batch, dtype=dtype, out_dtype=c_dtype, entry="k_relu__partial",
                    c_name="mm", **mm_kw)
    m1["final"] = False
    shape = ([batch] if batch > 1 else []) + [M, N]
    n = math.prod(shape)
    if axis_form:
        b = ("axis", "bias", (len(shape) - 1,))
        tile = shape
    else:
        b = ("bcast", "bias", N, 1, N)
        tile = None
    expr = ("add", "mm", b) if bias else "mm"
    if relu:
        expr = ("relu", expr)
    if expr == "mm":
        expr = ("copy", "mm")
    k2, m2 = pointwise(n, expr, compute, shape=shape, entry="k_relu", tile_shape=tile,
                       dtypes={"mm": c_dtype, "bias": "f32"}, out_dtype=out_dtype,
                       seeds={"bias": 2})
    for a in m2["args"]:
        if a["name"] == "mm":
            a["intermediate"] = True
            a.pop("seed", None)
    return [(k1, m1), (k2, m2)]


_ACC_NODES = {"Accum", "WarpShuffle", "TreeHalve", "Smem", "Init"}


def retype(kop, meta, dtype, acc=None):
    """The same IR over ``dtype`` tensors: every f32 type in the statements and
    every f32 argument becomes ``dtype``; accumulators and the combine
    statements that move them (Accum, WarpShuffle, TreeHalve, Smem, Init)
    become ``acc`` (default ``dtype``).  ``acc="f32"`` over ``dtype="f16"``
    is the f16 tensor / f32 accumulator form; ``acc="f16"`` rounds every fold
    to f16."""
    import dataclasses
    acc = acc or dtype
    to_t, to_a = DT[dtype], DT[acc]

    def walk(o, target):
        if isinstance(o, DataType):
            return target if o.name == "f32" else o
        if isinstance(o, tuple):
            return tuple(walk(v, target) for v in o)
        if dataclasses.is_dataclass(o) and not isinstance(o, type):
            t = to_a if type(o).__name__ in _ACC_NODES else target
            fields = {}
            for f in dataclasses.fields(o):
                v = getattr(o, f.name)
                if f.name == "dtype" and v == "float":          # shared buffers name C types
                    fields[f.name] = {"f32": "float", "f64": "double", "f16": "half"}[t.name]
                else:
                    fields[f.name] = walk(v, t)
            return dataclasses.replace(o, **fields)
        return o

    new = walk(kop, to_t)
    m = dict(meta)
    m["args"] = [dict(a, dtype=dtype) if a["dtype"] == "f32" else dict(a) for a in meta["args"]]
    return new, m
