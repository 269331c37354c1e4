"""GPU parity of integer pointwise programs (``emmy_pointwise_int``), bit for bit.

* Every integer program of ``oracle/make_ref_ptx.py`` (``INT_CASES``): the
  unmodified reference compiler's PTX, run on this GPU, the B200 kernel and
  the oracle give the same bits on the same inputs.  This pins the oracle's
  integer semantics to the reference itself.
* The same three-way check with float operands at the edges of the
  conversion (NaN, +-inf, beyond the s64 range, f16 and f64 inputs).
* Every op on every integer dtype against the oracle, shifts included (the
  reference's PTX for an integer shift Assign does not assemble, so the
  oracle's PTX-operand reading is the only bar there).
* A broadcast input, unaligned pointers (the element-at-a-time path) and a
  2^26 + 3 element run against numpy.
"""

from __future__ import annotations

import numpy as np
import pytest

from emmy_ir import synth
from gpu_util import run_on_gpu
from oracle import ref_ptx
from oracle.interp import run_ir
from oracle.make_ref_ptx import INT_CASES

pytestmark = pytest.mark.gpu

INT_DTS = ["i8", "u8", "i16", "u16", "i32", "u32", "i64", "u64"]
NZ = ("where", ("equal", "x1", ("imm", 0)), ("imm", 7), "x1")
OPS = ["add", "subtract", "multiply", "divide", "remainder", "left_shift", "right_shift",
       "bitwise_xor", "maximum", "minimum"]


def _bits(a):
    return np.ascontiguousarray(a).reshape(-1).view(np.uint8)


def _three_way(name, host=None):
    if not ref_ptx.available(name):
        pytest.skip("oracle/_ref not generated")
    kop, meta = INT_CASES[name](synth)
    host = host if host is not None else synth.make_inputs(meta)
    plan, _, ours = run_on_gpu(kop, meta, host)
    assert plan["family"] == "pointwise_int"
    k = ref_ptx.RefKernel(name)
    try:
        ref = k.run(host)
    finally:
        k.close()
    orc = run_ir(kop, meta, host)
    assert ours["out"].dtype == ref["out"].dtype
    assert np.array_equal(_bits(ours["out"]), _bits(ref["out"])), f"{name}: B200 vs reference PTX"
    assert np.array_equal(_bits(orc["out"]), _bits(ref["out"])), f"{name}: oracle vs reference PTX"


@pytest.mark.parametrize("name", sorted(INT_CASES))
def test_reference_ptx_b200_and_oracle_agree_bit_for_bit(name):
    _three_way(name)


def test_float_operand_edges_agree_with_the_reference_ptx():
    kop, meta = INT_CASES["I_float_in_i32"](synth)
    host = synth.make_inputs(meta)
    edges = [np.nan, np.inf, -np.inf, 1e30, -1e30, 2.0 ** 63, -(2.0 ** 63), 2.0 ** 31,
             -(2.0 ** 31) - 256.0, -2.75, 2.75, -0.5, 0.5, -0.0, 16777217.0, 3e9]
    host["x1"][:len(edges)] = np.array(edges, dtype=np.float32)
    _three_way("I_float_in_i32", host)
    kop, meta = INT_CASES["I_f16_f64_in_i64"](synth)
    host = synth.make_inputs(meta)
    with np.errstate(over="ignore"):
        host["x0"][:6] = np.array([np.nan, np.inf, -np.inf, 65504.0, -0.75, 2.5], np.float16)
    host["x1"][:6] = [1e300, -1e300, np.nan, 9.3e18, -9.3e18, 2.0 ** 62]
    _three_way("I_f16_f64_in_i64", host)


@pytest.mark.parametrize("dt", INT_DTS)
@pytest.mark.parametrize("op", OPS)
def test_op_matches_oracle(op, dt):
    expr = (op, "x0", NZ) if op in ("divide", "remainder") else (op, "x0", "x1")
    inits = None
    if op in ("left_shift", "right_shift"):
        inits = {"x1": {"dist": "int", "low": 0 if dt.startswith("u") else -70, "high": 70}}
    kop, meta = synth.pointwise(4099, expr, dt, inits=inits)
    host = synth.make_inputs(meta)
    _, _, out = run_on_gpu(kop, meta, host)
    want = run_ir(kop, meta, host)["out"]
    assert np.array_equal(_bits(out["out"]), _bits(want)), f"{op}/{dt}"


@pytest.mark.parametrize("out_dt", ["f16", "f32", "f64", "u8", "i64"])
def test_every_output_type(out_dt):
    kop, meta = synth.pointwise(4099, ("multiply", "x0", "x1"), "i64", out_dtype=out_dt,
                                inits={"x0": {"dist": "int", "low": -(1 << 40), "high": 1 << 40},
                                       "x1": {"dist": "int", "low": -5000, "high": 5000}})
    host = synth.make_inputs(meta)
    _, _, out = run_on_gpu(kop, meta, host)
    assert np.array_equal(_bits(out["out"]), _bits(run_ir(kop, meta, host)["out"]))


def test_broadcast_input():
    n, m = 4096 * 3, 64
    kop, meta = synth.pointwise(n, ("add", "x0", ("bcast", "b", m, 1, m)), "i32",
                                dtypes={"b": "i16"})
    host = synth.make_inputs(meta)
    plan, _, out = run_on_gpu(kop, meta, host)
    assert "input_index" in plan["pointwise"]
    want = (host["x0"].astype(np.int64) + np.tile(host["b"].astype(np.int64), n // m)).astype(np.int32)
    assert np.array_equal(out["out"], want)


def test_unaligned_pointers_take_the_element_path():
    import torch
    from ptxc import Lowerer
    from ptxc.launch import run
    n = 10001
    kop, meta = synth.pointwise(n, ("bitwise_xor", ("multiply", "x0", "x1"), "x0"), "i32")
    plan = Lowerer(kop, meta).plan()
    host = synth.make_inputs(meta)
    dev = torch.device("cuda:0")
    bufs = {k: torch.zeros(n + 1, dtype=torch.int32, device=dev) for k in ("x0", "x1", "out")}
    for k in ("x0", "x1"):
        bufs[k][1:] = torch.from_numpy(host[k]).to(dev)
    views = {k: v[1:] for k, v in bufs.items()}          # 4-byte offset: no 16-byte vectors
    run(plan, views)
    torch.cuda.synchronize()
    x, y = host["x0"].astype(np.int64), host["x1"].astype(np.int64)
    want = (((x * y) & 0xFFFFFFFF) ^ (x & 0xFFFFFFFF)).astype(np.uint32).view(np.int32)
    assert np.array_equal(views["out"].cpu().numpy(), want)
    assert int(bufs["out"][0]) == 0                       # nothing written before the view


def test_large_run_bit_exact():
    n = (1 << 26) + 3
    kop, meta = synth.pointwise(n, ("add", "x0", "x1"), "i32", unroll=1)
    host = synth.make_inputs(meta)
    _, _, out = run_on_gpu(kop, meta, host)
    with np.errstate(over="ignore"):
        assert np.array_equal(out["out"], host["x0"] + host["x1"])   # int32 wraps


def test_bench_program_full_size_matches_reference_ptx():
    """F8d (2^26 i32 adds, the bench line): B200 kernel = reference PTX = numpy, bit for bit."""
    from oracle.make_ref_ptx import BENCH_CASES
    name = "F8d_pointwise_int"
    if not ref_ptx.available(name):
        pytest.skip("oracle/_ref not generated")
    kop, meta = BENCH_CASES[name](synth)
    host = synth.make_inputs(meta)
    _, _, ours = run_on_gpu(kop, meta, host)
    k = ref_ptx.RefKernel(name)
    try:
        ref = k.run(host)
    finally:
        k.close()
    assert np.array_equal(ours["out"], ref["out"])
    with np.errstate(over="ignore"):
        assert np.array_equal(ours["out"], host["x0"] + host["x1"])


@pytest.mark.parametrize("expr", [
    # step 3 reads steps 1 and 2
    ("multiply", ("add", "x0", "x1"), ("subtract", "x0", "x1")),
    # five inputs
    ("add", ("add", ("add", ("add", "x0", "x1"), "x2"), "x3"), "x4"),
    # compare, where and remainder over three leaves
    ("remainder", ("where", ("less", "x0", "x1"), "x1", "x0"), NZ),
])
@pytest.mark.parametrize("dt", ["i16", "u32", "i64"])
def test_program_shapes_match_oracle(expr, dt):
    kop, meta = synth.pointwise(4099, expr, dt)
    host = synth.make_inputs(meta)
    _, _, out = run_on_gpu(kop, meta, host)
    assert np.array_equal(_bits(out["out"]), _bits(run_ir(kop, meta, host)["out"]))


WIDTH_CASES = [
    (("add", "x0", "x1"), "i32", {}),
    (("maximum", ("subtract", "x0", "x1"), ("imm", 0)), "u8", {}),
    (("add", "x0", "x1"), "u16", {"out_dtype": "i64"}),
    (("add", "x0", "x1"), "u16", {"out_dtype": "f16"}),
    (("where", ("greater", ("multiply", "x0", "x1"), ("imm", 0)), "x0", "x1"), "i16", {}),
    (("divide", "x0", ("imm", 3)), "i16", {}),
    (("divide", "x0", ("imm", -1)), "i16", {}),
    (("right_shift", "x0", "x1"), "i32", {}),
    (("left_shift", "x0", "x1"), "i64", {"out_dtype": "i32"}),
    (("multiply", ("add", "x0", "x1"), ("bitwise_xor", "x0", ("imm", -5))), "u32", {}),
    (("add", "x0", "x1"), "i32", {"dtypes": {"x1": "f32"},
                                  "inits": {"x1": {"dist": "uniform", "low": -3e9, "high": 3e9}}}),
]


@pytest.mark.parametrize("expr,dt,kw", WIDTH_CASES)
def test_32_bit_programs_store_the_64_bit_bits(expr, dt, kw):
    """Programs the matcher runs on 32-bit values: the same program forced to
    64 bits gives the same stored bits, inputs at their types' extremes included."""
    import copy
    import torch
    from ptxc import Lowerer
    from ptxc.launch import Executor
    kop, meta = synth.pointwise(4099, expr, dt, **kw)
    plan = Lowerer(kop, meta).plan()
    assert plan["pointwise"]["value_bits"] == 32
    host = synth.make_inputs(meta)
    for name, arr in host.items():
        if arr.dtype.kind in "iu" and name != "out":
            info = np.iinfo(arr.dtype)
            arr[:6] = [info.min, info.max, 0, -1 if arr.dtype.kind == "i" else 1, info.min + 1,
                       info.max - 1]
    outs = []
    for bits in (32, 64):
        p = copy.deepcopy(plan)
        p["pointwise"]["value_bits"] = bits
        ex = Executor(p)
        ex.upload(host)
        ex.launch()
        torch.cuda.synchronize()
        outs.append(ex.download()["out"].numpy())
    assert np.array_equal(_bits(outs[0]), _bits(outs[1]))
    assert np.array_equal(_bits(outs[0]), _bits(run_ir(kop, meta, host)["out"]))


@pytest.mark.parametrize("expr,dt", [
    # one op over inputs, then steps with a constant (clamps, scales, offsets)
    (("add", ("multiply", "x0", "x1"), ("imm", 3)), "i32"),
    (("subtract", ("imm", 100), ("bitwise_xor", "x0", "x1")), "i16"),            # swapped tail
    (("maximum", ("minimum", ("subtract", "x0", "x1"), ("const", "hi", 100)), ("imm", -100)), "i32"),
    (("remainder", ("add", ("multiply", "x0", ("imm", 5)), ("imm", -7)), ("imm", 9)), "i64"),
    (("divide", ("add", "x0", "x1"), ("imm", 3)), "u8"),
    (("left_shift", ("add", "x0", "x1"), ("imm", 3)), "u16"),
])
def test_op_then_constant_steps_match_oracle(expr, dt):
    kop, meta = synth.pointwise(4099, expr, dt)
    host = synth.make_inputs(meta)
    _, _, out = run_on_gpu(kop, meta, host)
    assert np.array_equal(_bits(out["out"]), _bits(run_ir(kop, meta, host)["out"]))


# ---- chain programs (the staged kernel) ---------------------------------------

def _is_chain(pw):
    """The library's rule for the staged chain kernel: each step reads only the
    step before it besides inputs and constants, and the last step is the result."""
    nleaf = len(pw["inputs"]) + len(pw["scalars"]) + len(pw["immediates"])
    writer = {}
    prog = pw["program"]
    if len(prog) < 2 or not pw["inputs"]:
        return False
    for k, (op, dst, *ops) in enumerate(prog):
        arity = 3 if op == 20 else 1 if op in (0, 19) else 2
        for r in ops[:arity]:
            if r >= nleaf and writer.get(r) != k - 1:
                return False
        writer[dst] = k
    return pw["result_reg"] >= nleaf and writer.get(pw["result_reg"]) == len(prog) - 1


CHAIN_CASES = [
    # (expr, dtype, kwargs)
    (("maximum", ("subtract", "x0", "x1"), ("imm", 0)), "u8", {}),
    (("bitwise_xor", ("right_shift", ("multiply", "x0", "x1"), ("imm", 3)), "x2"), "i32", {}),
    (("where", ("greater", ("subtract", "x0", "x1"), ("const", "t", 5)), "x1", "x0"), "i16", {}),
    (("add", ("multiply", "x0", ("imm", 3)), "x1"), "i64", {}),
    (("minimum", ("add", "x0", "x1"), ("imm", 1000)), "i32",
     {"dtypes": {"x1": "f32"}, "inits": {"x1": {"dist": "uniform", "low": -3e9, "high": 3e9}}}),
    (("left_shift", ("add", "x0", "x1"), ("imm", 2)), "u16", {"out_dtype": "f16"}),
    (("remainder", ("add", ("multiply", "x0", ("imm", 5)), ("imm", -7)), ("imm", 9)), "i64", {}),
    (("add", ("add", ("add", ("add", "x0", "x1"), "x2"), "x3"), "x4"), "u32", {}),
]


@pytest.mark.parametrize("n", [1024, 4096 * 3 + 5, (1 << 21) + 3])
@pytest.mark.parametrize("expr,dt,kw", CHAIN_CASES)
def test_chain_programs_match_oracle(expr, dt, kw, n):
    kop, meta = synth.pointwise(n, expr, dt, unroll=1, **kw)
    from ptxc import Lowerer
    assert _is_chain(Lowerer(kop, meta).plan()["pointwise"])
    host = synth.make_inputs(meta)
    _, _, out = run_on_gpu(kop, meta, host)
    assert np.array_equal(_bits(out["out"]), _bits(run_ir(kop, meta, host)["out"])), (expr, dt, n)


def test_chain_bench_program_full_size():
    """F8e (u8 max(x0 - x1, 0), 2^26 + 3 elements): many chunks per CTA, a tail."""
    n = (1 << 26) + 3
    kop, meta = synth.pointwise(n, ("maximum", ("subtract", "x0", "x1"), ("imm", 0)), "u8",
                                unroll=1)
    host = synth.make_inputs(meta)
    _, _, out = run_on_gpu(kop, meta, host)
    want = np.maximum(host["x0"].astype(np.int64) - host["x1"].astype(np.int64), 0).astype(np.uint8)
    assert np.array_equal(out["out"], want)


def test_chain_with_unaligned_output():
    """Inputs on 16-byte boundaries (staged), the output one element off (scalar stores)."""
    import torch
    from ptxc import Lowerer
    from ptxc.launch import run
    n = 3 * 1024 + 7
    kop, meta = synth.pointwise(n, ("maximum", ("subtract", "x0", "x1"), ("imm", 0)), "i32",
                                unroll=1)
    plan = Lowerer(kop, meta).plan()
    host = synth.make_inputs(meta)
    dev = torch.device("cuda:0")
    ins = {k: torch.from_numpy(host[k]).to(dev) for k in ("x0", "x1")}
    obuf = torch.full((n + 1,), -1, dtype=torch.int32, device=dev)
    run(plan, {**ins, "out": obuf[1:]})
    torch.cuda.synchronize()
    want = np.maximum(host["x0"].astype(np.int64) - host["x1"].astype(np.int64), 0).astype(np.int32)
    assert np.array_equal(obuf[1:].cpu().numpy(), want)
    assert int(obuf[0]) == -1


@pytest.mark.parametrize("n", [1001, 4096 * 2 + 9])
@pytest.mark.parametrize("dt", ["i8", "u8", "i16", "u16"])
def test_narrow_one_step_programs(dt, n):
    """One-step programs over 1- and 2-byte elements: the staged kernel from one
    chunk up, the one-step kernel below it."""
    for expr in (("add", "x0", "x1"), ("maximum", "x0", ("imm", 7)), ("bitwise_xor", "x0", "x1")):
        kop, meta = synth.pointwise(n, expr, dt, unroll=1)
        host = synth.make_inputs(meta)
        _, _, out = run_on_gpu(kop, meta, host)
        assert np.array_equal(_bits(out["out"]), _bits(run_ir(kop, meta, host)["out"])), (expr, dt, n)
