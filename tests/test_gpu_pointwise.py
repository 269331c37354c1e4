"""GPU parity of the pointwise family (``emmy_pointwise``).

* the reference's 17 pointwise fixtures, rebuilt with the synthesiser
  (``tests/golden/replicas.py``), against the reference's stored goldens with
  each fixture's own rtol/atol (0/0 where the reference demands bit-exact);
* every opcode in f32, f16 and f64 against the statement-level IR interpreter
  (``oracle.interp``) on 4099 elements (a ragged tail after the 4-wide groups);
* a 2**26 + 3 element add and a multiply-add chain, bit-exact against numpy;
* inputs and output at odd element offsets (the one-element-per-thread path).

Tolerances (per element, written here): ops that are correctly rounded in IEEE
arithmetic (add, subtract, multiply, divide, sqrt, reciprocal, fma, min, max,
neg, abs, relu, floor, ceil, sign, comparisons, where) must match exactly;
transcendentals ``|d| <= 1e-5*|ref| + 1e-6`` in f32 (the fixtures' own bound),
``1e-12*|ref| + 1e-15*max|ref|`` in f64 (the absolute term covers the
cancellation in ``1 + erf(x)`` for negative x); f16 results within one f16 ulp
(``2e-3*|ref| + 2e-3``, the fixtures allow 1e-2).
"""

from __future__ import annotations

import numpy as np
import pytest

from emmy_ir import synth
from golden import replicas
from gpu_util import assert_close, run_on_gpu
from oracle.interp import run_ir
from ptxc.match_pointwise import ARITY, COMPARES, OPCODES, UNARY

pytestmark = pytest.mark.gpu

EXACT = {"copy", "add", "subtract", "multiply", "divide", "maximum", "minimum", "negative", "abs",
         "sqrt", "reciprocal", "relu", "floor", "ceil", "sign", "where"} | COMPARES
POSITIVE = {"log", "sqrt", "rsqrt", "log2", "log10", "pow"}


@pytest.mark.parametrize("fid", [f for f in replicas.replica_ids() if "_p_" in f])
def test_fixture_replica_matches_reference_golden(fid):
    kop, meta, names = replicas.build(fid)
    plan, host, out = run_on_gpu(kop, meta, replicas.fixture_inputs(fid, meta, names))
    assert plan["family"] == "pointwise"
    worst, msg = replicas.compare(fid, out[replicas.table()[fid]["output"]])
    assert worst <= 0, msg


def _op_case(op, dt):
    ar = ARITY.get(op, 1 if op in UNARY else 2)
    expr = (op, *["x0", "x1", "x2"][:ar])
    if op in COMPARES:
        expr = ("where", expr, "x0", "x1")
    inits = None
    if op in POSITIVE:
        inits = {"x0": {"dist": "uniform", "low": 0.05, "high": 4.0},
                 "x1": {"dist": "uniform", "low": -3.0, "high": 3.0}}
    return synth.pointwise(4099, expr, dt, inits=inits)


OPS = [op for op in OPCODES if op != "round_f16"]


@pytest.mark.parametrize("dt", ["f32", "f16", "f64"])
@pytest.mark.parametrize("op", OPS)
def test_opcode_matches_interpreter(op, dt):
    kop, meta = _op_case(op, dt)
    host = synth.make_inputs(meta)
    plan, _, out = run_on_gpu(kop, meta, host)
    ref = run_ir(kop, meta, host)["out"].astype(np.float64)
    got = out["out"].astype(np.float64)
    if dt == "f16":
        exact = op in EXACT and op != "divide"
        rtol, atol = (0.0, 0.0) if exact else (2e-3, 2e-3)
    elif op in EXACT or op == "fma":
        rtol, atol = 0.0, 0.0
    else:
        rtol, atol = (1e-5, 1e-6) if dt == "f32" else (1e-12, 1e-15 * float(np.abs(ref).max()))
    fin = np.isfinite(ref)
    assert np.array_equal(fin, np.isfinite(got)), f"{op}/{dt}: inf/nan positions differ"
    assert_close(got[fin], ref[fin], rtol, atol, f"{op}/{dt}")


def test_large_add_bit_exact():
    n = (1 << 26) + 3
    kop, meta = synth.pointwise(n, ("add", "x0", "x1"), "f32", unroll=1)
    host = synth.make_inputs(meta)
    _, _, out = run_on_gpu(kop, meta, host)
    assert np.array_equal(out["out"], host["x0"] + host["x1"])


def test_large_chain_bit_exact():
    n = 3 * (1 << 24)
    expr = ("add", ("multiply", ("const", "scale", 1.5), "x0"), ("divide", "x1", ("imm", 3.0)))
    kop, meta = synth.pointwise(n, expr, "f32")
    host = synth.make_inputs(meta)
    _, _, out = run_on_gpu(kop, meta, host)
    want = np.float32(1.5) * host["x0"] + host["x1"] / np.float32(3.0)
    assert np.array_equal(out["out"], want)


def test_unaligned_offsets_use_scalar_path():
    import torch
    from ptxc import Lowerer
    from ptxc.launch import run
    n = 10001
    kop, meta = synth.pointwise(n, ("subtract", ("multiply", "x0", "x1"), "x0"), "f32")
    plan = Lowerer(kop, meta).plan()
    host = synth.make_inputs(meta)
    dev = torch.device("cuda:0")
    bufs = {k: torch.zeros(n + 1, dtype=torch.float32, device=dev) for k in ("x0", "x1", "out")}
    for k in ("x0", "x1"):
        bufs[k][1:] = torch.from_numpy(host[k]).to(dev)
    views = {k: v[1:] for k, v in bufs.items()}          # 4-byte offset: not 16-byte aligned
    run(plan, views)
    torch.cuda.synchronize()
    got = views["out"].cpu().numpy()
    assert np.array_equal(got, host["x0"] * host["x1"] - host["x0"])
    assert float(bufs["out"][0]) == 0.0                   # nothing written before the view


def test_gelu_f16_whole_groups_matches_general_path_and_float64():
    """f16 gelu (tanh form) on whole 8-element groups runs the packed 16-byte
    kernel; one more 4-element group sends the same values through the
    general f16 path.  Both within one f16 ulp (2e-3 * |ref| + 2e-3, as the
    opcode test) of each other and of float64."""
    n = 1 << 20
    kop, meta = synth.pointwise(n, ("gelu_tanh", "x0"), "f16")
    host = synth.make_inputs(meta)
    _, _, out = run_on_gpu(kop, meta, host)
    kop2, meta2 = synth.pointwise(n + 4, ("gelu_tanh", "x0"), "f16")
    host2 = synth.make_inputs(meta2)
    host2["x0"][:n] = host["x0"]
    _, _, out2 = run_on_gpu(kop2, meta2, host2)
    got = out["out"].astype(np.float64)
    general = out2["out"][:n].astype(np.float64)
    x = host["x0"].astype(np.float64)
    ref = 0.5 * x * (1.0 + np.tanh(np.sqrt(2.0 / np.pi) * (x + 0.044715 * x ** 3)))
    assert_close(got, general, 2e-3, 2e-3, "packed vs general f16 path")
    assert_close(got, ref, 2e-3, 2e-3, "packed f16 path vs float64")
    assert np.mean(got == general) > 0.99
