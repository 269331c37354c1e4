"""Scalar semantics probe for the family matcher.

The matcher decides what a run of ``Let``/``Load``/``Assign``/``Accum``
statements computes (an accumulator update, a cross-thread combine, an
epilogue) by evaluating those statements on a few random float64 points and
comparing with each family's closed form.  This accepts every spelling of the
same formula (operand order, temporaries, names) and rejects any other
formula with overwhelming probability; it never runs the kernel or touches
tensors.  Op meanings are the reference's elementwise table
(``ptxc/expr.py:880-1089``, ``ptxc/ops.py:81-96``).
"""

from __future__ import annotations

import math

from .common import CompileError, op_name, stmt_name


class ProbeMismatch(Exception):
    pass


def _op(opname: str, args: list):
    a = args[0] if args else None
    b = args[1] if len(args) > 1 else None
    try:
        if opname in ("add", "sum"):
            return a + b
        if opname in ("subtract", "sub"):
            return a - b
        if opname in ("multiply", "prod"):
            return a * b
        if opname in ("divide", "true_divide", "divide_rn_f32"):
            return a / b
        if opname in ("maximum", "amax", "max"):
            return max(a, b)
        if opname in ("minimum", "min"):
            return min(a, b)
        if opname in ("exp", "exp_fast"):
            return math.exp(a) if a > -700 else 0.0
        if opname == "exp2":
            return 2.0 ** a
        if opname == "log":
            return math.log(a)
        if opname == "sqrt":
            return math.sqrt(a)
        if opname == "rsqrt":
            return 1.0 / math.sqrt(a)
        if opname == "reciprocal":
            return 1.0 / a
        if opname == "relu":
            return max(a, 0.0)
        if opname in ("copy", "pad", "bitcast"):
            return a
        if opname in ("negative", "negate"):
            return -a
        if opname in ("abs", "fabs"):
            return abs(a)
        if opname == "tanh":
            return math.tanh(a)
        if opname == "fma":
            return a * b + args[2]
        if opname in ("greater", "gt"):
            return 1.0 if a > b else 0.0
        if opname in ("less", "lt"):
            return 1.0 if a < b else 0.0
        if opname == "where":
            return args[1] if a else args[2]
    except (ValueError, ZeroDivisionError, OverflowError) as exc:
        raise ProbeMismatch(str(exc)) from exc
    raise ProbeMismatch(f"op {opname!r}")


def run_scalar(stmts, env: dict, load=None, accum_rule=None) -> dict:
    """Evaluate straight-line scalar statements in place on ``env`` (name -> float).

    ``load(st)`` returns the values of a ``Load`` (one per name).  ``Accum``
    folds ``op(base or acc, value)`` into ``env[name]``.  Any other statement
    raises ``ProbeMismatch``.
    """
    for st in stmts:
        kind = stmt_name(st)
        if kind == "Let":
            v = getattr(st.value, "value", st.value)
            env[st.name] = float(v)
        elif kind == "Load":
            if load is None:
                raise ProbeMismatch("load outside a probe")
            vals = load(st)
            for n, v in zip(st.names, vals):
                env[n] = v
        elif kind == "Assign":
            args = []
            for a in st.args:
                if isinstance(a, (int, float)) and not isinstance(a, bool):
                    args.append(float(a))
                elif a in env:
                    args.append(env[a])
                else:
                    raise ProbeMismatch(f"undefined {a!r}")
            env[st.name] = _op(op_name(st.op), args)
        elif kind == "Accum":
            if st.name not in env:
                raise ProbeMismatch(f"unseeded accumulator {st.name!r}")
            left = env[st.base] if st.base is not None else env[st.name]
            if st.base is not None and st.base not in env:
                raise ProbeMismatch("undefined base")
            if st.value not in env:
                raise ProbeMismatch("undefined value")
            env[st.name] = _op(op_name(st.op), [left, env[st.value]])
        elif kind in ("Sync", "Smem"):
            continue
        else:
            raise ProbeMismatch(f"statement {kind} in a scalar probe")
    return env


def close(a: float, b: float, rel: float = 1e-9) -> bool:
    if math.isnan(a) or math.isnan(b):
        return False
    return abs(a - b) <= rel * max(1.0, abs(a), abs(b))


def probe(points, fn_ir, fn_ref, rel: float = 1e-9) -> bool:
    """True when ``fn_ir(p)`` matches ``fn_ref(p)`` (tuples of floats) at every point."""
    for p in points:
        try:
            got = fn_ir(p)
        except (ProbeMismatch, KeyError):
            return False
        want = fn_ref(p)
        if len(got) != len(want):
            return False
        if not all(close(g, w, rel) for g, w in zip(got, want)):
            return False
    return True


def require(cond: bool, msg: str) -> None:
    if not cond:
        raise CompileError(msg)
