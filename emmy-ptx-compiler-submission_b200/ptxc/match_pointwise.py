"""Family matcher for the pointwise (elementwise) IR shape.

Shape (reference fixtures ``v_p_*``, ``w_p_*``; lowering in
``ptxc/stmts.py:73-145`` (Load), ``:434-487`` (Write), ``ptxc/expr.py:880-1089``
(elementwise ops)):

    Tile(a0 : T)                       -- or no axis for a single element
      [U unrolled copies, element e = U*a0 + u:]
        Load in_i[e] ...; Load c[0] ...  -- tensors and one-element constants
        Assign v = op(...) ...
      Write out[U*a0 (+u)] = values     -- one vector write or U scalar writes

Every written element must be the same expression of the same tensors, each
read at that element's own index (checked copy by copy), and the writes must
cover the output exactly once (``T*U == numel``).  The expression becomes a
small register program (``program``) that ``emmy_pointwise`` evaluates per
element.
"""

from __future__ import annotations

import math

from .affine import Affine, broadcast_form, decode_axes, flat_affine
from .common import norm_dtype, op_name, stmt_name
from .match_reduce import NoMatch, need

# opcode table shared with csrc/pointwise.cu (the reference's float op table,
# ptxc/ops.py:81-96 and ptxc/expr.py:880-1089, plus the comparisons and
# ``round_f16``, which re-rounds an f16-typed result)
OPCODES = {
    "copy": 0, "add": 1, "subtract": 2, "multiply": 3, "divide": 4, "maximum": 5,
    "minimum": 6, "negative": 7, "abs": 8, "exp": 9, "log": 10, "sqrt": 11, "rsqrt": 12,
    "reciprocal": 13, "tanh": 14, "sigmoid": 15, "relu": 16, "greater": 17, "less": 18,
    "greater_equal": 19, "less_equal": 20, "equal": 21, "where": 22, "round_f16": 23,
    "fma": 24, "log2": 25, "log10": 26, "cos": 27, "sin": 28, "tan": 29, "erf": 30,
    "gelu": 31, "gelu_tanh": 32, "softplus": 33, "exp2": 34, "silu": 35, "pow": 36,
    "floor": 37, "ceil": 38, "sign": 39, "not_equal": 40,
}
ALIASES = {"sum": "add", "sub": "subtract", "prod": "multiply", "true_divide": "divide",
           "divide_rn_f32": "divide", "amax": "maximum", "max": "maximum", "min": "minimum",
           "negate": "negative", "fabs": "abs", "gt": "greater", "lt": "less",
           "ge": "greater_equal", "le": "less_equal", "eq": "equal", "ne": "not_equal", "exp_fast": "exp",
           "pad": "copy", "bitcast": "copy"}
ARITY = {"where": 3, "fma": 3}
UNARY = {"copy", "negative", "abs", "exp", "log", "sqrt", "rsqrt", "reciprocal", "tanh",
         "sigmoid", "relu", "round_f16", "log2", "log10", "cos", "sin", "tan", "erf", "gelu",
         "gelu_tanh", "softplus", "exp2", "silu", "floor", "ceil", "sign"}
COMPARES = {"greater", "less", "greater_equal", "less_equal", "equal", "not_equal"}
MAX_REGS = 32
MAX_INSTR = 48


def match_pointwise(kop, tile, meta) -> dict:
    shapes, dtypes = meta.shapes, meta.dtypes
    axes = [(a.name, int(a.extent.value)) for a in tile.axes]
    rename = None
    if len(axes) > 1:
        # a multi-axis Tile: each axis is a decode of the flat work id "__g"
        rename = decode_axes(axes)
        T, avar = math.prod(e for _, e in axes), "__g"
    else:
        T = axes[0][1] if axes else 1
        avar = axes[0][0] if axes else None
    stmts = list(tile.body)
    need(stmts, "empty Tile")
    for st in stmts:
        need(stmt_name(st) in ("Load", "Assign", "Let", "Write"), f"{stmt_name(st)} in a pointwise body")
    writes = [st for st in stmts if stmt_name(st) == "Write"]
    need(writes, "no write")
    outs = {w.output for w in writes}
    need(len(outs) == 1, "writes to several outputs")
    out = outs.pop()
    need(out in shapes and not any(w.atomic for w in writes), "output buffer")
    numel = math.prod(shapes[out]) if shapes[out] else 1

    defs = {}       # name -> ("load", tensor, affine) | ("let", value) | ("op", opname, args, dtype)
    for st in stmts:
        k = stmt_name(st)
        if k == "Load":
            need(st.input in shapes, f"load of unknown buffer {st.input!r}")
            aff = flat_affine(st.index, shapes[st.input], rename, keep_atoms=True)
            need(aff is not None, "non-affine pointwise index")
            for i, nm in enumerate(st.names):
                a2 = Affine(aff)
                a2[""] = a2.get("", 0) + i
                defs[nm] = ("load", st.input, a2)
        elif k == "Let":
            defs[st.name] = ("let", float(getattr(st.value, "value", st.value)))
        elif k == "Assign":
            op = ALIASES.get(op_name(st.op), op_name(st.op))
            need(op in OPCODES, f"no pointwise kernel op for {op!r}")
            need(len(st.args) == ARITY.get(op, 1 if op in UNARY else 2), f"{op} arity")
            defs[st.name] = ("op", op, tuple(st.args), norm_dtype(st.dtype) if st.dtype else None)

    # written elements: (offset affine, value name)
    elems = []
    for w in writes:
        aff = flat_affine(w.index, shapes[out], rename)
        need(aff is not None, "non-affine output index")
        for i, v in enumerate(w.values):
            a2 = dict(aff)
            a2[""] = a2.get("", 0) + i
            elems.append((a2, v))
    coef = {tuple(sorted((k, c) for k, c in a.items() if k)) for a, _ in elems}
    need(len(coef) == 1, "output elements use different index strides")
    var_part = dict(next(iter(coef)))
    U = var_part.get(avar, 0) if avar else 0
    need(set(var_part) <= ({avar} if avar else set()), "output index uses a non-Tile variable")
    offs = sorted(a.get("", 0) for a, _ in elems)
    if avar and T > 1:
        need(U == len(elems) and offs == list(range(U)), "writes do not tile the output")
    else:
        need(offs == list(range(len(elems))), "writes do not tile the output")
    need(max(T, 1) * max(len(elems), 1) == numel or (not avar and len(elems) == numel),
         "writes do not cover the output exactly once")

    # canonical per-element program, checked equal for every element
    inputs, scalars, imms = [], [], []

    def canon(name, elem_aff, memo, depth=0):
        need(depth < 64, "pointwise expression too deep")
        if name in memo:
            return memo[name]
        d = defs.get(name)
        need(d is not None, f"undefined value {name!r}")
        if d[0] == "let":
            r = ("imm", d[1])
        elif d[0] == "load":
            tensor, aff = d[1], d[2]
            tn = math.prod(shapes[tensor]) if shapes[tensor] else 1
            bc = None if aff.atoms_ok() else broadcast_form(aff)
            if tn == 1 and not {k for k, c in aff.items() if k and c} and aff.get("", 0) == 0:
                r = ("scalar", tensor)
            elif not aff.atoms_ok():
                # broadcast: the element's own offset E, read at (E // D) % M
                need(bc is not None, f"{tensor!r} index is neither the element nor a broadcast of it")
                E, D, M = bc
                need({k: c for k, c in E.items() if c} == {k: c for k, c in elem_aff.items() if c},
                     f"{tensor!r} is not a broadcast of the written element")
                top = min(M - 1, (numel - 1) // D) if M else (numel - 1) // D
                need(top < tn, f"{tensor!r} broadcast reads past its {tn} elements")
                r = ("input", (tensor, D, M))
            else:
                rel = {k: c for k, c in aff.items() if c}
                want = {k: c for k, c in elem_aff.items() if c}
                need(rel == want, f"{tensor!r} is not read at the written element")
                need(tn == numel, f"{tensor!r} does not match the output size")
                r = ("input", (tensor, 0, 0))
        else:
            r = ("op", d[1], tuple(canon(a, elem_aff, memo, depth + 1) for a in d[2]), d[3])
        memo[name] = r
        return r

    forms = [canon(v, a, {}) for a, v in elems]
    need(all(f == forms[0] for f in forms), "elements compute different expressions")
    form = forms[0]

    # lower the expression tree to a register program
    prog = []

    def leaf_reg(kind, key):
        # registers are numbered once the leaf counts are known (reg_of below)
        lst = {"input": inputs, "scalar": scalars, "imm": imms}[kind]
        if key not in lst:
            lst.append(key)
        return (kind, key)

    def emit(node):
        if node[0] in ("input", "scalar", "imm"):
            return leaf_reg(node[0], node[1])
        _, op, args, dt = node
        srcs = [emit(a) for a in args]
        prog.append([op, srcs])
        ref = ("tmp", len(prog) - 1)
        if dt == "f16" and op not in COMPARES:
            prog.append(["round_f16", [ref]])
            ref = ("tmp", len(prog) - 1)
        return ref

    result = emit(form)
    if (prog and prog[-1][0] == "round_f16" and dtypes[out] == "f16"
            and result == ("tmp", len(prog) - 1)):
        # the f16 store rounds once; rounding to f16 twice gives the same value
        src = prog.pop()[1][0]
        result = src
    if result[0] != "tmp":
        prog.append(["copy", [result]])
        result = ("tmp", len(prog) - 1)
    base = {"input": 0, "scalar": len(inputs), "imm": len(inputs) + len(scalars)}
    ntmp0 = len(inputs) + len(scalars) + len(imms)

    def reg_of(ref):
        if ref[0] == "tmp":
            return ntmp0 + ref[1]
        lst = {"input": inputs, "scalar": scalars, "imm": imms}[ref[0]]
        return base[ref[0]] + lst.index(ref[1])

    program = []
    for i, (op, srcs) in enumerate(prog):
        rs = [reg_of(s) for s in srcs] + [0] * (3 - len(srcs))
        program.append([OPCODES[op], ntmp0 + i] + rs)
    need(ntmp0 + len(prog) <= MAX_REGS and len(prog) <= MAX_INSTR, "pointwise program too large")

    in_index = [[D, M] for _, D, M in inputs]
    inputs = [t for t, _, _ in inputs]
    in_dts = {dtypes[t] for t in inputs + scalars}
    need(in_dts <= {"f32", "f16", "f64"} and dtypes[out] in ("f32", "f16", "f64"),
         "pointwise dtypes must be f16/f32/f64")
    compute = "f64" if ("f64" in in_dts or dtypes[out] == "f64") else "f32"
    return {
        "family": "pointwise", "symbol": "emmy_pointwise",
        "args": {"out": out},
        "pointwise": {"n": numel, "inputs": inputs, "scalars": scalars, "immediates": imms,
                      "program": program, "result_reg": ntmp0 + len(prog) - 1,
                      "compute": compute, "out_dtype": dtypes[out],
                      **({"input_index": in_index, "first": 0}
                         if any(D for D, _ in in_index) else {})},
        "params": {}, "dtypes": {"out": dtypes[out]},
    }
