"""Affine analysis of IR index expressions.

An index coordinate built from ``Var``, integer ``Literal``, ``+``, ``-`` and
multiplication by a constant is affine in the Tile axes and loop variables.
The flat element offset of a load or write is then
``sum_i coord_i * stride_i`` with the row-major strides of the reference's
``_strides`` rule: as many strides as coordinates, taken from the declared
shape, and a lone coordinate is already flat (``ptxc/common.py:398-415``,
``ptxc/memory.py:150-186``).  The matcher reads tensor layouts (row, column
and batch strides) off these forms.
"""

from __future__ import annotations

from .common import const_int


class Affine(dict):
    """``{var: coefficient}`` plus the constant under key ``""``."""

    def const(self) -> int:
        return self.get("", 0)

    def coef(self, var: str) -> int:
        return self.get(var, 0)

    def vars(self) -> set:
        return {k for k, v in self.items() if k and v}

    def atoms_ok(self) -> bool:
        return all(isinstance(k, str) for k, v in self.items() if v)

    def key(self) -> tuple:
        return tuple(sorted((k, v) for k, v in self.items() if v))


def _add(a: Affine, b: Affine, sign: int = 1) -> Affine:
    out = Affine(a)
    for k, v in b.items():
        out[k] = out.get(k, 0) + sign * v
    return out


def _scale(a: Affine, s: int) -> Affine:
    return Affine({k: v * s for k, v in a.items()})


def affine_of(e, rename=None):
    """Affine form of an index expression, or None when it is not affine."""
    name = type(e).__name__
    if e is None:
        return None
    if name == "Var" or name == "Builtin":
        v = e.name
        if rename and v in rename:
            v = rename[v]
        return Affine({v: 1})
    if name in ("Literal", "Dim") or isinstance(e, int):
        c = const_int(e)
        if c is None:
            return None
        return Affine({"": c})
    if name == "BinaryExpr":
        left = affine_of(e.left, rename)
        right = affine_of(e.right, rename)
        if left is None or right is None:
            return None
        if e.op in ("+", "add"):
            return _add(left, right)
        if e.op in ("-", "subtract"):
            return _add(left, right, -1)
        if e.op in ("*", "multiply"):
            if not left.vars():
                return _scale(right, left.const())
            if not right.vars():
                return _scale(left, right.const())
            return None
        if e.op in ("/", "//", "divide", "floor_divide", "%", "mod", "remainder"):
            # (E // c) and (E % c) of an affine E stay symbolic atoms; a flat
            # index that holds c*k*(E//c) + k*(E%c) recombines to k*E below.
            c = right.const() if not right.vars() else None
            if c is None or c <= 0 or not left.atoms_ok():
                return None
            kind = "div" if e.op in ("/", "//", "divide", "floor_divide") else "mod"
            return Affine({(kind, _frozen(left), c): 1})
        return None
    return None


def _frozen(a: Affine) -> tuple:
    return tuple(sorted(((k, v) for k, v in a.items() if v), key=repr))


def _recombine(a: Affine):
    out = Affine(a)
    for key in list(out):
        if isinstance(key, tuple) and key[0] == "div" and out.get(key):
            mod = ("mod", key[1], key[2])
            k2 = out.get(mod, 0)
            if k2 and out[key] == key[2] * k2:
                del out[key]
                del out[mod]
                out = _add(out, _scale(Affine(dict(key[1])), k2))
    if not out.atoms_ok():
        return None
    return out


def strides_of(shape, ncoords: int) -> list:
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


def flat_affine(index, shape, rename=None):
    """Affine flat element offset of ``buffer[index]`` for a buffer of ``shape``."""
    if index is None or len(index) == 0:
        return Affine({"": 0})
    if len(index) == 1:
        a = affine_of(index[0], rename)
        return None if a is None else _recombine(a)
    acc = Affine()
    for coord, stride in zip(index, strides_of(shape, len(index))):
        a = affine_of(coord, rename)
        if a is None:
            return None
        acc = _add(acc, _scale(a, stride))
    return _recombine(acc)
