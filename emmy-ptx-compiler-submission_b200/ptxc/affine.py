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
            if isinstance(v, Affine):       # an axis standing for a decoded flat id
                return Affine(v)
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
            # (E // c) and (E % c) of an affine E (itself possibly holding
            # such atoms) stay symbolic atoms; a flat index that holds
            # c*k*(E//c) + k*(E%c) recombines to k*E below.
            c = right.const() if not right.vars() else None
            if c is None or c <= 0:
                return None
            if e.op in ("/", "//", "divide", "floor_divide"):
                return Affine({_div_key(left, c): 1})
            return Affine({("mod", _frozen(left), c): 1})
        return None
    return None


def _frozen(a: Affine) -> tuple:
    return tuple(sorted(((k, v) for k, v in a.items() if v), key=repr))


def _div_key(left: Affine, c: int) -> tuple:
    """The atom ``left // c``, with ``(E // a) // c`` kept as ``E // (a*c)``
    (equal for non-negative E), so every quotient of E has one spelling."""
    ks = [k for k, v in left.items() if v]
    if len(ks) == 1 and isinstance(ks[0], tuple) and ks[0][0] == "div" and left[ks[0]] == 1:
        return ("div", ks[0][1], ks[0][2] * c)
    return ("div", _frozen(left), c)


def _recombine(a: Affine, keep_atoms: bool = False):
    """Fold every ``c*k*(E//c) + k*(E%c)`` pair into ``k*E``, repeatedly (a
    multi-axis decode nests them).  Atoms left over make the form non-affine:
    None, unless ``keep_atoms``."""
    out = Affine(a)
    changed = True
    while changed:
        changed = False
        for key in list(out):
            if isinstance(key, tuple) and key[0] == "mod" and out.get(key):
                k2 = out[key]
                left = Affine(dict(key[1]))
                div = _div_key(left, key[2])
                if out.get(div, 0) == key[2] * k2:
                    del out[key]
                    del out[div]
                    out = _add(out, _scale(left, k2))
                    changed = True
                    break
    out = Affine({k: v for k, v in out.items() if v or k == ""})
    if not keep_atoms and not out.atoms_ok():
        return None
    return out


def decode_axes(axes, flat: str = "__g") -> dict:
    """Each Tile axis as a form of the flat work id, as the reference decodes
    it: ``idx_i = (gid / suffix_i) % extent_i`` (``ptxc/lower.py:787-812``),
    written as nested divisions so that the flat index of a row-major load
    recombines to the flat id.  The first axis needs no ``%`` (the gid guard
    keeps it in range)."""
    out = {}
    cur = Affine({flat: 1})
    for i in range(len(axes) - 1, -1, -1):
        name, ext = axes[i]
        if i == 0:
            out[name] = Affine(cur)
        else:
            out[name] = Affine({("mod", _frozen(cur), int(ext)): 1})
            cur = Affine({_div_key(cur, int(ext)): 1})
    return out


def broadcast_form(a: Affine):
    """``(E, D, M)`` when the offset ``a`` is ``(E // D) % M`` (``M = 0``: no
    ``%``; ``D = 1``: no ``//``) of an atom-free affine ``E``, else None."""
    keys = [k for k, v in a.items() if v and k != ""]
    if a.const() or len(keys) != 1 or not isinstance(keys[0], tuple) or a[keys[0]] != 1:
        return None
    kind, left, c = keys[0]
    D, M = 1, 0
    if kind == "mod":
        M = c
        inner = Affine(dict(left))
    else:
        inner = Affine({keys[0]: 1})
    ks = [k for k, v in inner.items() if v and k != ""]
    if len(ks) == 1 and isinstance(ks[0], tuple) and ks[0][0] == "div" \
            and inner[ks[0]] == 1 and not inner.const():
        D = ks[0][2]
        inner = Affine(dict(ks[0][1]))
    if not inner.atoms_ok():
        return None
    return inner, D, M


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


def flat_affine(index, shape, rename=None, keep_atoms=False):
    """Affine flat element offset of ``buffer[index]`` for a buffer of ``shape``
    (``keep_atoms``: also return forms with ``//`` / ``%`` atoms left over)."""
    if index is None or len(index) == 0:
        return Affine({"": 0})
    if len(index) == 1:
        a = affine_of(index[0], rename)
        return None if a is None else _recombine(a, keep_atoms)
    acc = Affine()
    for coord, stride in zip(index, strides_of(shape, len(index))):
        a = affine_of(coord, rename)
        if a is None:
            return None
        acc = _add(acc, _scale(a, stride))
    return _recombine(acc, keep_atoms)
