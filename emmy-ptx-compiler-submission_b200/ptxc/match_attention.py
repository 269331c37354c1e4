"""Family matcher for the attention-like matmul -> softmax -> reduce IR shape.

Shape (reference fixtures ``v_a_*``, ``w_a_*``; the reference lowers it
statement by statement: ``ptxc/stmts.py:663-725`` for the key and head-dim
loops, ``:1311-1392`` for its warp-cooperative dot, ``:564-611`` for the
rescaled online accumulators, ``ptxc/expr.py:891-895`` for exp):

    Tile(... query-row and value-column axes ...)
      Load div -> v1 = recip(div)                         (the score scale)
      Loop over keys a1 (or a lane-strided StridedLoop):
        Loop over head dim a2 { Load q[row, a2]; Load k[a1, a2] (or kt[a2, a1]);
                                multiply; Accum add }      -- one per register row
        s = dot * v1; online (max, sum, sum of p * v[a1, col]) with exp rescale
      [WarpShuffle / TreeHalve combine of (max, sum, weighted sum) across lanes]
      Write out[row, col] = weighted sum * recip(sum)

The matcher checks this signature: the head-dim dot loops (two global loads,
a product, an add fold), which operand moves with the key variable (k) and
which does not (q), the value load indexed by the key, an online max
accumulator and two rescaled add accumulators over the key axis, the scale as
the reciprocal of a one-element constant, and a final write of
``weighted_sum * recip(sum)`` reaching every output element.  Layouts (whether k is
stored pre-transposed) come from the affine forms of the k and v indices;
shapes from meta.json.  Row/column register tiling may index q and the output
with wrapped (``%``) expressions, so their coverage is checked by count, not
by address.
"""

from __future__ import annotations

import math

from .affine import affine_of
from .common import const_int, norm_dtype, op_name, stmt_name
from .match_reduce import NoMatch, need


def _walk(stmts, parents=()):
    for st in stmts:
        yield st, parents
        for attr in ("body", "else_body"):
            child = getattr(st, attr, None)
            if isinstance(child, (tuple, list)) and child:
                yield from _walk(child, parents + (st,))


def _is_dot_loop(st, shapes):
    if stmt_name(st) != "Loop":
        return False
    body = list(st.body)
    loads = [s for s in body if stmt_name(s) == "Load"]
    muls = [s for s in body if stmt_name(s) == "Assign" and op_name(s.op) == "multiply"]
    accs = [s for s in body if stmt_name(s) == "Accum"]
    if len(body) != 4 or len(loads) != 2 or len(muls) != 1 or len(accs) != 1:
        return False
    if any(l.input not in shapes or len(l.names) != 1 for l in loads):
        return False
    names = {l.names[0] for l in loads}
    return (set(muls[0].args) == names and accs[0].value == muls[0].name
            and op_name(accs[0].op) == "add" and accs[0].base is None)


def match_attention(kop, tile, meta) -> dict:
    shapes, dtypes = meta.shapes, meta.dtypes
    walked = list(_walk(tile.body))
    dots = [(st, par) for st, par in walked if _is_dot_loop(st, shapes)]
    need(dots, "no head-dim dot-product loop")
    dvar = dots[0][0].axis.name
    D = int(dots[0][0].axis.extent.value)
    need(all(st.axis.name == dvar and int(st.axis.extent.value) == D for st, _ in dots),
         "dot loops disagree on the head dim")
    key_loops = {id(par[-1]): par[-1] for _, par in dots if par}
    need(len(key_loops) == 1, "dot loops are not inside one key loop")
    kl = next(iter(key_loops.values()))
    need(stmt_name(kl) in ("Loop", "StridedLoop"), "key loop kind")
    kvar = kl.axis.name
    Sk = int(kl.axis.extent.value)

    # q and k operands
    q_name = k_name = None
    k_trans = None
    for st, _ in dots:
        for l in (s for s in st.body if stmt_name(s) == "Load"):
            idx = tuple(l.index)
            uses_key = any(kvar in getattr(c, "free_vars", lambda: frozenset())() for c in idx)
            if uses_key:
                need(k_name in (None, l.input), "several key operands")
                k_name = l.input
                need(len(idx) >= 2, "key operand index rank")
                a_last, a_prev = affine_of(idx[-1]), affine_of(idx[-2])
                if a_last is not None and a_prev is not None and a_last.key() == ((dvar, 1),) \
                        and a_prev.vars() == {kvar} and a_prev.coef(kvar) == 1:
                    t = False                       # k[..., key, d]
                elif a_last is not None and a_prev is not None and a_prev.key() == ((dvar, 1),) \
                        and a_last.vars() == {kvar} and a_last.coef(kvar) == 1:
                    t = True                        # kt[..., d, key]
                else:
                    raise NoMatch("key operand index is neither k[key, d] nor kt[d, key]")
                need(k_trans in (None, t), "key operand read in two layouts")
                k_trans = t
            else:
                need(q_name in (None, l.input), "several query operands")
                q_name = l.input
                a_last = affine_of(idx[-1])
                need(a_last is not None and a_last.key() == ((dvar, 1),),
                     "query operand is not indexed [row, d]")
    need(q_name and k_name and q_name != k_name, "query/key operands")

    # value operand, online accumulators
    v_name = None
    acc_max, acc_add_base = set(), set()
    dot_ids = {id(st) for st, _ in dots}
    for st in kl.body:
        if id(st) in dot_ids:
            continue
        k = stmt_name(st)
        if k == "Load":
            need(st.input in shapes, "unknown load in the key loop")
            idx = tuple(st.index)
            a_prev = affine_of(idx[-2]) if len(idx) >= 2 else None
            need(a_prev is not None and a_prev.vars() == {kvar} and a_prev.coef(kvar) == 1,
                 "value operand is not indexed [key, col]")
            need(v_name in (None, st.input), "several value operands")
            v_name = st.input
        elif k == "Accum":
            need(tuple(st.axes or ())[:1] == (kvar,), "accumulator not over the key axis")
            if op_name(st.op) == "maximum":
                need(st.base is None, "max accumulator with a base")
                acc_max.add(st.name)
            elif op_name(st.op) == "add":
                need(st.base is not None, "sum accumulator without the rescale base")
                acc_add_base.add(st.name)
            else:
                raise NoMatch("unexpected fold in the key loop")
        elif k not in ("Assign", "Let"):
            raise NoMatch(f"{k} in the key loop")
    need(v_name is not None and v_name not in (q_name, k_name), "no value operand")
    need(acc_max and len(acc_add_base) == 2 * len(acc_max), "online softmax accumulators")
    for st in kl.body:
        if stmt_name(st) == "Assign" and op_name(st.op) == "exp":
            break
    else:
        raise NoMatch("no exp rescale in the key loop")

    # scale: recip of a one-element constant multiplied into the score
    consts = [st.input for st, _ in walked if stmt_name(st) == "Load" and st.input in shapes
              and math.prod(shapes[st.input] or (1,)) == 1]
    scale_name = None
    if consts:
        need(len(set(consts)) == 1, "several scalar constants")
        scale_name = consts[0]
        loaded = {n for st, _ in walked if stmt_name(st) == "Load" and st.input == scale_name
                  for n in st.names}
        recips = {st.name for st, _ in walked if stmt_name(st) == "Assign"
                  and op_name(st.op) == "reciprocal" and set(st.args) <= loaded}
        dot_accs = {next(s.name for s in st.body if stmt_name(s) == "Accum") for st, _ in dots}
        scaled = [st for st, _ in walked if stmt_name(st) == "Assign" and op_name(st.op) == "multiply"
                  and set(st.args) & recips and set(st.args) & dot_accs]
        need(recips and scaled, "the score scale is not dot * recip(constant)")

    # final writes: weighted_sum * recip(sum)
    writes = [st for st, _ in walked if stmt_name(st) == "Write" and st.output in shapes]
    need(writes, "no output write")
    outs = {w.output for w in writes}
    need(len(outs) == 1, "writes to several outputs")
    o_name = outs.pop()
    need(not any(w.atomic for w in writes), "atomic attention output")
    assigns = {st.name: st for st, _ in walked if stmt_name(st) == "Assign"}
    for w in writes:
        need(len(w.values) == 1, "vector output write")
        val = assigns.get(w.values[0])
        need(val is not None and op_name(val.op) == "multiply", "output is not a product")
        rec = [assigns.get(a) for a in val.args]
        need(any(r is not None and op_name(r.op) == "reciprocal" for r in rec),
             "output does not divide by the softmax sum")

    # shapes and coverage
    qs, ks, vs, os_ = shapes[q_name], shapes[k_name], shapes[v_name], shapes[o_name]
    need(len(qs) >= 2 and len(qs) == len(ks) == len(vs) == len(os_), "operand ranks")
    lead = qs[:-2]
    need(ks[:-2] == lead and vs[:-2] == lead and os_[:-2] == lead, "batch dims differ")
    Sq, Dq = qs[-2], qs[-1]
    if k_trans:
        Dk, Sk2 = ks[-2], ks[-1]
    else:
        Sk2, Dk = ks[-2], ks[-1]
    Sv, Dv = vs[-2], vs[-1]
    need(Dq == Dk == D and Sk2 == Sv == Sk, "q/k/v shapes do not chain")
    need(os_[-2] == Sq and os_[-1] == Dv, "output shape")
    lanes = math.prod(int(a.extent.value) for a in tile.axes)
    coop = [a for a in tile.axes if a.name.endswith("_co")]
    rows_written = lanes // (math.prod(int(a.extent.value) for a in coop) if coop else 1)
    # register tiling may wrap rows (``% S``) and recompute a few of them, so
    # the writes must reach every element at least once
    need(rows_written * len(writes) >= math.prod(os_), "writes do not cover the output")
    batch = math.prod(lead) if lead else 1

    dts = {dtypes[q_name], dtypes[k_name], dtypes[v_name]}
    need(len(dts) == 1, "q/k/v dtypes differ")
    dt = dts.pop()
    odt = dtypes[o_name]
    g = {"batch": batch, "sq": Sq, "sk": Sk, "d": D, "dv": Dv, "k_transposed": bool(k_trans)}
    args = {"q": q_name, "k": k_name, "v": v_name, "o": o_name}
    if scale_name:
        args["scale"] = scale_name
    if dt == "f32":
        need(odt == "f32", "f32 attention with a non-f32 output")
        return {"family": "attention_f32", "symbol": "emmy_attention_f32", "args": args,
                "attention": g, "params": {}, "dtypes": {"qkv": dt, "o": odt}}
    if dt == "f16":
        need(odt in ("f16", "f32"), "f16 attention output must be f16 or f32")
        g["out_dtype"] = 1 if odt == "f16" else 0
        return {"family": "attention_f16", "symbol": "emmy_attention_f16", "args": args,
                "attention": g, "params": {}, "dtypes": {"qkv": dt, "o": odt}}
    raise NoMatch(f"no B200 attention kernel for {dt}")
