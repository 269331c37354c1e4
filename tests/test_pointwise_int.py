"""Integer pointwise programs on the CPU: the oracle, the matcher, the C-ABI checks.

The reference lowers integer-typed pointwise Assigns on signed 64-bit
registers (``ptxc/stmts.py:509-560``, ``ptxc/ops.py:98-117``,
``ptxc/expr.py:157-223, 697-716, 815-877, 233-280``).  Here:

* the oracle's integer path (``oracle.interp``) against a restatement of
  those rules in plain Python integers, op by op and dtype by dtype;
* the float <-> integer conversions (cvt.rzi.s64 saturating with NaN -> -2^63,
  cvt.rn.f32.s64 correctly rounded, f16 through f32);
* the matcher's integer plans and its refusals, with the reference's messages;
* ``emmy_pointwise_int``'s host-side argument checks (no GPU needed);
* when the reference checkout is present, that its compiler emitted PTX for
  every integer program the GPU tests run it on.
"""

from __future__ import annotations

import ctypes
import json
from fractions import Fraction

import numpy as np
import pytest

from conftest import PKG, ROOT
from emmy_ir import synth
from oracle.interp import run_ir
from oracle.make_ref_ptx import INT_CASES

INT_DTS = ["i8", "u8", "i16", "u16", "i32", "u32", "i64", "u64"]
M64 = 1 << 64
NZ = ("where", ("equal", "x1", ("imm", 0)), ("imm", 7), "x1")


def s64(x):
    x &= M64 - 1
    return x - M64 if x >> 63 else x


def tdiv(a, b):
    q = abs(a) // abs(b)
    return q if (a < 0) == (b < 0) else -q


PY_OPS = {
    "add": lambda a, b: s64(a + b),
    "subtract": lambda a, b: s64(a - b),
    "multiply": lambda a, b: s64(a * b),
    "divide": lambda a, b: tdiv(a, b),
    "remainder": lambda a, b: a - tdiv(a, b) * b,
    "left_shift": lambda a, b: 0 if (b & 0xFFFFFFFF) >= 64 else s64(a << (b & 0xFFFFFFFF)),
    "right_shift": lambda a, b: ((-1 if a < 0 else 0) if (b & 0xFFFFFFFF) >= 64
                                 else a >> (b & 0xFFFFFFFF)),
    "bitwise_xor": lambda a, b: a ^ b,
    "maximum": max,
    "minimum": min,
}


def as_s64(arr):
    return [s64(int(v)) for v in arr.tolist()]


def store(values, dt):
    """The low bits of each s64 value, as dtype dt."""
    width = np.dtype(synth.NP[dt]).itemsize * 8
    u = np.array([v & ((1 << width) - 1) for v in values], dtype=np.uint64)
    return u.astype(np.dtype(f"u{width // 8}") if width < 64 else np.uint64).view(synth.NP[dt])


@pytest.mark.parametrize("dt", INT_DTS)
@pytest.mark.parametrize("op", sorted(PY_OPS))
def test_oracle_integer_op_matches_python_integers(op, dt):
    if op in ("divide", "remainder"):
        expr = (op, "x0", NZ)
    else:
        expr = (op, "x0", "x1")
    inits = None
    if op in ("left_shift", "right_shift"):
        lo = 0 if dt.startswith("u") else -70
        inits = {"x1": {"dist": "int", "low": lo, "high": 70}}
    kop, meta = synth.pointwise(257, expr, dt, inits=inits)
    host = synth.make_inputs(meta)
    got = run_ir(kop, meta, host)["out"]
    a, b = as_s64(host["x0"]), as_s64(host["x1"])
    if op in ("divide", "remainder"):
        b = [7 if v == 0 else v for v in b]
    want = store([PY_OPS[op](x, y) for x, y in zip(a, b)], dt)
    assert got.dtype == want.dtype and np.array_equal(got, want)


def test_oracle_predicates_where_and_the_and_or_quirk():
    # bitwise_and / bitwise_or are predicates in the reference's Assign: (a != 0) & (b != 0)
    kop, meta = synth.pointwise(
        1000, ("where", ("bitwise_or", ("bitwise_and", "x0", "x1"), ("less", "x0", ("imm", 0))),
               "x0", "x1"), "i8")
    host = synth.make_inputs(meta)
    host["x0"][:4] = [0, 5, -3, 0]
    host["x1"][:4] = [9, 0, 0, 0]
    got = run_ir(kop, meta, host)["out"]
    x, y = host["x0"].astype(np.int64), host["x1"].astype(np.int64)
    c = ((x != 0) & (y != 0)) | (x < 0)
    assert np.array_equal(got, np.where(c, x, y).astype(np.int8))
    assert got[:4].tolist() == [9, 0, -3, 0]


def test_oracle_float_operands_truncate_and_saturate():
    kop, meta = synth.pointwise(12, ("add", "x0", "x1"), "i64", dtypes={"x1": "f32"})
    host = synth.make_inputs(meta)
    host["x0"][:] = 0
    specials = [np.nan, np.inf, -np.inf, 1e30, -1e30, 2.0 ** 63, -(2.0 ** 63), -2.75, 2.75,
                -0.5, 16777217.0, 3e9]
    host["x1"][:] = np.array(specials, dtype=np.float32)
    got = run_ir(kop, meta, host)["out"].tolist()
    imax, imin = (1 << 63) - 1, -(1 << 63)
    assert got == [imin, imax, imin, imax, imin, imax, imin, -2, 2, 0, 16777216, 3000000000]


def test_oracle_float_outputs_round_like_cvt():
    kop, meta = synth.pointwise(8, ("add", "x0", ("imm", 0)), "i64", out_dtype="f32")
    host = synth.make_inputs(meta)
    vals = [2 ** 62 + 2 ** 38 + 1, -(2 ** 62 + 2 ** 38 + 1), 2 ** 24 + 1, 2 ** 24 + 3,
            (1 << 63) - 1, -(1 << 63), 123456789, -1]
    host["x0"][:] = vals
    got = run_ir(kop, meta, host)["out"]
    for g, v in zip(got.tolist(), vals):
        # correctly rounded: no f32 is nearer to v, ties to even
        f = Fraction(g)
        up = Fraction(float(np.nextafter(np.float32(g), np.float32(np.inf))))
        dn = Fraction(float(np.nextafter(np.float32(g), np.float32(-np.inf))))
        assert abs(f - v) <= abs(up - v) and abs(f - v) <= abs(dn - v), (v, g)
    # f16 output: through f32, as cvt.rn.f32.s64 then cvt.rn.f16.f32
    kop, meta = synth.pointwise(4, ("add", "x0", ("imm", 0)), "i64", out_dtype="f16")
    host = synth.make_inputs(meta)
    host["x0"][:] = [65519, 65520, 2049, -70000]
    got = run_ir(kop, meta, host)["out"]
    with np.errstate(over="ignore"):                               # -70000 -> -inf
        want = np.array([65519, 65520, 2049, -70000], np.int64).astype(np.float32).astype(np.float16)
    assert np.array_equal(got.view(np.uint16), want.view(np.uint16))


@pytest.mark.parametrize("name", sorted(INT_CASES))
def test_matcher_plans_every_reference_integer_case(name):
    from ptxc import Lowerer
    kop, meta = INT_CASES[name](synth)
    plan = Lowerer(kop, meta).plan()
    assert plan["family"] == "pointwise_int" and plan["symbol"] == "emmy_pointwise_int"
    g = plan["pointwise"]
    assert 1 <= len(g["program"]) <= 48 and all(len(r) == 5 for r in g["program"])
    assert all(isinstance(v, int) for v in g["immediates"])


@pytest.mark.parametrize("expr,dt,kw,needle", [
    (("negative", "x0"), "i32", {}, "unsupported integer op 'negative'"),
    (("abs", "x0"), "i64", {}, "unsupported integer op 'abs'"),
    (("greater", "x0", "x1"), "i32", {}, "cannot store a predicate value"),
    (("multiply", "x0", ("imm", 0.5)), "f32", {"dtypes": {"x0": "i32"}}, "float arithmetic"),
])
def test_matcher_refuses_what_the_reference_refuses(expr, dt, kw, needle):
    from ptxc import CompileError, Lowerer
    kop, meta = synth.pointwise(64, expr, dt, **kw)
    with pytest.raises(CompileError) as e:
        Lowerer(kop, meta).plan()
    assert needle in str(e.value)


def test_float_programs_stay_on_the_float_kernel():
    from ptxc import Lowerer
    kop, meta = synth.pointwise(64, ("add", "x0", ("imm", 1.5)), "f32")
    assert Lowerer(kop, meta).plan()["family"] == "pointwise"


@pytest.fixture(scope="module")
def lib():
    lib = ctypes.CDLL(str(PKG / "libemmyb200.so"))
    lib.emmy_last_error.restype = ctypes.c_char_p
    vp, i, i64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64
    lib.emmy_pointwise_int.argtypes = [vp, vp, vp, i, vp, vp, i, vp, i, vp, i, i, vp, i, i64, i64, i,
                                       vp]
    return lib


def _call(lib, program, *, n=64, in_dt=7, out_dt=7, index=None, result=None, imms=(), bits=64):
    ins = (ctypes.c_void_p * 2)(16, 32)
    dts = (ctypes.c_int * 2)(in_dt, in_dt)
    flat = [int(x) for row in program for x in row]
    prog = (ctypes.c_int * len(flat))(*flat)
    imm = (ctypes.c_int64 * max(1, len(imms)))(*imms)
    idx = (ctypes.c_int64 * 6)(*index) if index else None
    res = result if result is not None else 2 + len(imms) + len(program) - 1
    return lib.emmy_pointwise_int(ins, dts, idx, 2, None, None, 0, imm, len(imms), prog,
                                  len(program), res, ctypes.c_void_p(48), out_dt, 0, n, bits, None)


def test_capi_host_checks_need_no_gpu(lib):
    assert _call(lib, [[1, 2, 0, 1, 0]], n=0) == 0                 # nothing to do
    assert _call(lib, [[21, 2, 0, 1, 0]]) == 1
    assert b"unknown opcode" in lib.emmy_last_error()
    assert _call(lib, [[1, 0, 0, 1, 0]]) == 1                      # writes an input register
    assert b"writes register" in lib.emmy_last_error()
    assert _call(lib, [[1, 2, 0, 1, 0]], bits=16) == 1
    assert b"value_bits" in lib.emmy_last_error()
    assert _call(lib, [[1, 2, 0, 1, 0]], out_dt=11) == 1
    assert b"bad output dtype" in lib.emmy_last_error()
    assert _call(lib, [[1, 2, 0, 1, 0]], in_dt=-1) == 1
    assert b"bad input dtype" in lib.emmy_last_error()
    assert _call(lib, [[1, 2, 0, 1, 0]], result=7) == 1
    assert b"bad result register" in lib.emmy_last_error()
    # a broadcast input read at e % 65 with only 64 elements
    assert _call(lib, [[1, 2, 0, 1, 0]], n=200, index=[1, 65, 64, 0, 0, 0]) == 1
    assert b"read past" in lib.emmy_last_error()


def test_reference_compiled_every_integer_case():
    report = ROOT / "oracle" / "_ref" / "report.json"
    if not report.exists():
        pytest.skip("no reference PTX here (oracle/_ref is made where the reference checkout is)")
    rep = json.loads(report.read_text())
    for name in INT_CASES:
        assert rep.get(name, {}).get("rc") == 0, (name, rep.get(name))
        assert (ROOT / "oracle" / "_ref" / name / "kernel.ptx").exists()


@pytest.mark.parametrize("expr,dt,kw,bits", [
    (("add", "x0", "x1"), "i32", {}, 32),                       # low bits only
    (("maximum", ("subtract", "x0", "x1"), ("imm", 0)), "u8", {}, 32),   # exact, in range
    (("add", "x0", "x1"), "i32", {"out_dtype": "f32"}, 64),     # exact, 2^32 wide
    (("add", "x0", "x1"), "u16", {"out_dtype": "i64"}, 32),     # exact, in range
    (("maximum", "x0", "x1"), "u32", {}, 64),                   # u32 does not fit int32
    (("greater", ("multiply", "x0", "x1"), ("imm", 0)), "i16", {"out_dtype": "i8"}, None),
    (("where", ("greater", ("multiply", "x0", "x1"), ("imm", 0)), "x0", "x1"), "i16", {}, 32),
    (("where", ("greater", ("multiply", "x0", "x1"), ("imm", 0)), "x0", "x1"), "i32", {}, 64),
    (("divide", "x0", ("imm", 3)), "i16", {}, 32),
    (("divide", "x0", ("imm", -1)), "i32", {}, 64),              # INT32_MIN / -1
    (("remainder", "x0", "x1"), "i16", {}, 64),                  # the divisor may be 0
    (("right_shift", "x0", "x1"), "i32", {}, 32),
    (("right_shift", "x0", "x1"), "u32", {}, 64),
    (("left_shift", "x0", "x1"), "i64", {}, 64),                  # an i64 output is exact
    (("left_shift", "x0", "x1"), "i64", {"out_dtype": "i32"}, 32),  # its low 32 bits only
])
def test_value_bits_proof(expr, dt, kw, bits):
    """The matcher's choice of 32-bit evaluation on small programs."""
    from ptxc import CompileError, Lowerer
    kop, meta = synth.pointwise(64, expr, dt, **kw)
    if bits is None:                                   # a predicate stored: refused
        with pytest.raises(CompileError):
            Lowerer(kop, meta).plan()
        return
    got = Lowerer(kop, meta).plan()["pointwise"]["value_bits"]
    assert got == bits, (expr, dt, got)
