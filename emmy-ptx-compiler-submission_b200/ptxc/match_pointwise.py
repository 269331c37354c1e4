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
            v = getattr(st.value, "value", st.value)
            need(isinstance(v, (int, float)) and not isinstance(v, bool), "Let of a non-literal")
            defs[st.name] = ("let", v, norm_dtype(st.dtype) if st.dtype else "f32")
        elif k == "Assign":
            defs[st.name] = ("op", op_name(st.op), tuple(st.args),
                             norm_dtype(st.dtype) if st.dtype else None)

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
            r = ("imm", d[1], d[2])
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
    if _is_integer_program(form, dtypes, out):
        return _lower_integer(form, dtypes, out, numel)

    # lower the expression tree to a register program
    prog = []

    def leaf_reg(kind, key):
        # registers are numbered once the leaf counts are known (reg_of below)
        lst = {"input": inputs, "scalar": scalars, "imm": imms}[kind]
        if key not in lst:
            lst.append(key)
        return (kind, key)

    def emit(node):
        if node[0] == "imm":
            return leaf_reg("imm", float(node[1]))
        if node[0] in ("input", "scalar"):
            return leaf_reg(node[0], node[1])
        _, op, args, dt = node
        op = ALIASES.get(op, op)
        need(op in OPCODES, f"no pointwise kernel op for {op!r}")
        need(len(args) == ARITY.get(op, 1 if op in UNARY else 2), f"{op} arity")
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


# ---------------------------------------------------------------------------
# Integer programs (reference ptxc/stmts.py:509-560 Assign, ptxc/ops.py:98-117
# INT_BINARY, ptxc/expr.py:815-877 predicates / where, :233-280 the store).
# The reference types each Assign by its dtype (or, untyped, by its first
# operand's kind): comparisons, and / or (``bitwise_and`` / ``bitwise_or``
# too) and typed-bool ops give predicates, float types go to the float path,
# every other op runs on s64.  A program with any integer value runs on the
# integer kernel (``emmy_pointwise_int``), whose opcodes are these:

INT_KINDS = {"i8", "u8", "i16", "u16", "i32", "u32", "i64", "u64"}
FLOAT_KINDS = {"f16", "f32", "f64"}
INT_OPCODES = {
    "copy": 0, "add": 1, "subtract": 2, "multiply": 3, "divide": 4, "remainder": 5,
    "left_shift": 6, "right_shift": 7, "bitwise_xor": 8, "maximum": 9, "minimum": 10,
    "equal": 11, "not_equal": 12, "greater": 13, "less": 14, "greater_equal": 15,
    "less_equal": 16, "and": 17, "or": 18, "not": 19, "where": 20,
}
INT_ALIASES = {"sum": "add", "sub": "subtract", "prod": "multiply", "floor_divide": "divide",
               "true_divide": "divide", "mod": "remainder", "amax": "maximum"}
CMP_ALIASES = {"eq": "equal", "ne": "not_equal", "gt": "greater", "lt": "less",
               "ge": "greater_equal", "le": "less_equal"}
BOOL_BINARY = {"bitwise_and": "and", "logical_and": "and", "and": "and",
               "bitwise_or": "or", "logical_or": "or", "or": "or"}
BOOL_NOT = {"bitwise_not", "logical_not", "not"}


def _leaf_kind(node, dtypes):
    if node[0] == "input":
        return dtypes[node[1][0]]
    if node[0] == "scalar":
        return dtypes[node[1]]
    return node[2]                                     # imm: the Let's dtype


def _kind(node, dtypes):
    """The reference's kind of a value: a dtype name, "i64" or "pred"."""
    if node[0] != "op":
        return _leaf_kind(node, dtypes)
    _, op, args, dt = node
    dt = dt or _kind(args[0], dtypes)
    if dt == "bool" or op in CMP_ALIASES or op in COMPARES or op in BOOL_BINARY:
        return "pred"
    if op == "where":
        return "f32" if (dt in FLOAT_KINDS or _kind(args[1], dtypes) in FLOAT_KINDS
                         or _kind(args[2], dtypes) in FLOAT_KINDS) else "i64"
    if dt in FLOAT_KINDS:
        return dt
    if op in ("copy", "pad", "bitcast"):
        return _kind(args[0], dtypes)
    return "i64"


def _is_integer_program(form, dtypes, out) -> bool:
    seen = []

    def walk(node):
        seen.append(_kind(node, dtypes))
        if node[0] == "op":
            for a in node[2]:
                walk(a)
    walk(form)
    return dtypes[out] in INT_KINDS or any(k in INT_KINDS or k == "i64" for k in seen)


def _rzi_f32(v) -> int:
    """A float literal as an s64 operand: its f32 value, truncated toward zero."""
    import numpy as np
    f = float(np.float32(v))
    need(math.isfinite(f) and abs(f) < 2.0 ** 63, "integer immediate out of range")
    return int(f)


def _lower_integer(form, dtypes, out, numel) -> dict:
    out_dt = dtypes[out]
    need(out_dt in INT_KINDS or out_dt in FLOAT_KINDS, f"output dtype {out_dt!r}")
    inputs, scalars, imms, prog = [], [], [], []

    def leaf(node):
        if node[0] == "imm":
            v = node[1]
            v = _rzi_f32(v) if isinstance(v, float) else int(v)
            v = (v + (1 << 63)) % (1 << 64) - (1 << 63)            # mov.s64 of the literal
            key, lst = ("imm", v), imms
        elif node[0] == "scalar":
            key, lst = ("scalar", node[1]), scalars
        else:
            key, lst = ("input", node[1]), inputs
        need(_leaf_kind(node, dtypes) in INT_KINDS | FLOAT_KINDS, "leaf dtype")
        if key[1] not in lst:
            lst.append(key[1])
        return key

    def operand(node, what):
        k = _kind(node, dtypes)
        need(k != "pred", f"a predicate used as an integer operand ({what})")
        need(node[0] != "op" or k not in FLOAT_KINDS, f"float arithmetic in an integer program ({what})")
        return emit(node)

    def cond(node):
        k = _kind(node, dtypes)
        need(node[0] != "op" or k not in FLOAT_KINDS, "float value as an integer predicate")
        need(k not in FLOAT_KINDS, "a float value tested in an integer program")
        return emit(node)

    def emit(node):
        if node[0] != "op":
            return leaf(node)
        _, op, args, dt = node
        k = _kind(node, dtypes)
        if op in ("copy", "pad", "bitcast"):
            need(len(args) == 1, f"{op} arity")
            return emit(args[0])                       # mov: the value, its kind kept
        if k == "pred":
            if op in BOOL_BINARY:
                need(len(args) == 2, f"{op} arity")
                name, srcs = BOOL_BINARY[op], [cond(args[0]), cond(args[1])]
            elif op in BOOL_NOT:
                need(len(args) == 1, f"{op} arity")
                name, srcs = "not", [cond(args[0])]
            else:
                name = CMP_ALIASES.get(op, op)
                need(name in COMPARES, f"unsupported boolean op {op!r}")
                need(len(args) == 2, f"{op} arity")
                need(not any(_kind(a, dtypes) in FLOAT_KINDS for a in args),
                     "comparison of float values in an integer program")
                srcs = [operand(args[0], op), operand(args[1], op)]
        elif k in FLOAT_KINDS:
            need(False, f"float arithmetic in an integer program ({op})")
        elif op == "where":
            need(len(args) == 3, "where arity")
            name, srcs = "where", [cond(args[0]), operand(args[1], op), operand(args[2], op)]
        else:
            name = INT_ALIASES.get(op, op)
            need(name in INT_OPCODES and name not in COMPARES and name not in ("and", "or", "not",
                                                                                 "where", "copy"),
                 f"unsupported integer op {op!r}")
            need(len(args) == 2, f"{op} arity")
            srcs = [operand(args[0], op), operand(args[1], op)]
        prog.append([name, srcs])
        return ("tmp", len(prog) - 1)

    need(_kind(form, dtypes) != "pred", "cannot store a predicate value as a scalar")
    result = emit(form)
    if result[0] != "tmp":
        prog.append(["copy", [result]])
        result = ("tmp", len(prog) - 1)
    in_keys = inputs
    leaf_dt = {("input", k): dtypes[k[0]] for k in in_keys}
    leaf_dt.update({("scalar", k): dtypes[k] for k in scalars})
    leaf_dt.update({("imm", v): v for v in imms})
    bits = value_bits(prog, result, leaf_dt, out_dt)
    base = {"input": 0, "scalar": len(in_keys), "imm": len(in_keys) + len(scalars)}
    ntmp0 = len(in_keys) + len(scalars) + len(imms)

    def reg_of(ref):
        if ref[0] == "tmp":
            return ntmp0 + ref[1]
        lst = {"input": in_keys, "scalar": scalars, "imm": imms}[ref[0]]
        return base[ref[0]] + lst.index(ref[1])

    program = []
    for i, (name, srcs) in enumerate(prog):
        rs = [reg_of(x) for x in srcs] + [0] * (3 - len(srcs))
        program.append([INT_OPCODES[name], ntmp0 + i] + rs)
    need(ntmp0 + len(prog) <= MAX_REGS and len(prog) <= MAX_INSTR, "pointwise program too large")
    need(len(in_keys) <= 8 and len(scalars) <= 8 and len(imms) <= 8, "pointwise program too large")
    in_index = [[D, M] for _, D, M in in_keys]
    names = [t for t, _, _ in in_keys]
    return {
        "family": "pointwise_int", "symbol": "emmy_pointwise_int",
        "args": {"out": out},
        "pointwise": {"n": numel, "inputs": names, "scalars": scalars, "immediates": imms,
                      "program": program, "result_reg": ntmp0 + len(prog) - 1,
                      "compute": "i64", "out_dtype": out_dt, "value_bits": bits,
                      **({"input_index": in_index, "first": 0}
                         if any(D for D, _ in in_index) else {})},
        "params": {}, "dtypes": {"out": out_dt},
    }


# ---------------------------------------------------------------------------
# 32-bit evaluation of an integer program.  The reference computes on s64.
# The same stored bits come out of 32-bit registers when every value that
# must be exact fits in int32 and every other value is used only through its
# low 32 bits:
#   * add, sub, mul, xor, shl and copy: the low 32 bits of the result depend
#     only on the low 32 bits of the operands (shl.b32 / shl.b64 both give 0
#     past their width, and both read the count's low 32 bits);
#   * comparisons, max, min, div, rem, shr's value, where's condition and the
#     logical ops read the whole value: their operands must be exact;
#   * the stored result must be exact for a float or 64-bit output, and only
#     its low bits count for an integer output of 32 bits or fewer.
# Exactness flows from the result and those operands down to the leaves;
# ranges flow up from the leaves' types and the immediates by interval
# arithmetic on unbounded integers.  A value that must be exact needs a range
# inside int32 (then no s64 operation on the way wrapped either).  A division
# or remainder counts as exact too: a zero divisor or INT32_MIN / -1 gives the
# 32-bit and 64-bit instructions different (unspecified) bits.

INT32_LO, INT32_HI = -(1 << 31), (1 << 31) - 1
DT_RANGE = {"i8": (-128, 127), "u8": (0, 255), "i16": (-32768, 32767), "u16": (0, 65535),
            "i32": (INT32_LO, INT32_HI), "u32": (0, (1 << 32) - 1),
            "i64": (-(1 << 63), (1 << 63) - 1), "u64": (-(1 << 63), (1 << 63) - 1)}
_LOW_BITS = {"add", "subtract", "multiply", "bitwise_xor", "copy", "left_shift"}


def _range_of(name, rs):
    """Interval of an instruction's result from its operands' intervals (None: unbounded)."""
    if any(r is None for r in rs):
        return None
    a = rs[0]
    b = rs[1] if len(rs) > 1 else None
    if name == "copy":
        return a
    if name == "add":
        return (a[0] + b[0], a[1] + b[1])
    if name == "subtract":
        return (a[0] - b[1], a[1] - b[0])
    if name == "multiply":
        p = [x * y for x in a for y in b]
        return (min(p), max(p))
    if name in ("divide", "remainder"):
        if b[0] <= 0 <= b[1]:
            return None                                    # a zero divisor is possible
        m = max(abs(a[0]), abs(a[1]))
        if name == "remainder":
            m = min(m, max(abs(b[0]), abs(b[1])) - 1)
        return (0 if a[0] >= 0 else -m, m)
    if name == "left_shift":
        if b[0] < 0 or b[1] > 62:
            return None
        p = [x << c for x in a for c in b]
        return (min(p), max(p))
    if name == "right_shift":
        return (min(a[0], 0), max(a[1], 0))                # toward 0 / -1 for any count
    if name == "bitwise_xor":
        if a[0] >= 0 and b[0] >= 0:
            return (0, (1 << max(a[1], b[1]).bit_length()) - 1)
        k = max(abs(v) for v in a + b).bit_length()
        return (-(1 << k), (1 << k) - 1)
    if name == "maximum":
        return (max(a[0], b[0]), max(a[1], b[1]))
    if name == "minimum":
        return (min(a[0], b[0]), min(a[1], b[1]))
    if name == "where":
        c = rs[2]
        return (min(b[0], c[0]), max(b[1], c[1]))
    return (0, 1)                                          # comparisons, and / or / not


def value_bits(prog, result, leaf_dtypes, out_dt) -> int:
    """32 when the program's stored bits are the same on 32-bit values, else 64.
    ``prog``: [(name, [ref...])] with refs ("tmp", i) or leaf keys; ``result``:
    the result ref; ``leaf_dtypes``: leaf ref -> dtype (ints, floats) or an int
    (an immediate's value)."""
    exact = set()
    if out_dt in FLOAT_KINDS or out_dt in ("i64", "u64"):
        exact.add(result)
    for i in range(len(prog) - 1, -1, -1):
        name, srcs = prog[i]
        mine = ("tmp", i) in exact
        if name in _LOW_BITS:
            if mine:
                exact.update(srcs[:1] if name == "left_shift" else srcs)
        elif name == "right_shift":
            exact.add(srcs[0])
        elif name == "where":
            exact.add(srcs[0])
            if mine:
                exact.update(srcs[1:])
        else:
            exact.update(srcs)
    ranges = {}

    def rng(ref):
        if ref[0] == "tmp":
            return ranges[ref]
        d = leaf_dtypes[ref]
        return (d, d) if isinstance(d, int) else DT_RANGE.get(d)

    for i, (name, srcs) in enumerate(prog):
        ranges[("tmp", i)] = _range_of(name, [rng(s) for s in srcs])
        if name in ("divide", "remainder"):
            # div.s32 / rem.s32 and the s64 forms agree only without a zero
            # divisor or an overflowing quotient: the result's own range (None
            # when the divisor may be 0) must lie inside int32
            exact.add(("tmp", i))
    for ref in exact:
        r = rng(ref)
        if r is None or r[0] < INT32_LO or r[1] > INT32_HI:
            return 64
    return 32
