"""Row families over f16 / f64 / mixed tensors (``emmy_rowop``) on the GPU.

The reference's dtype cases (``tools/specs/dtype_specs.py``: f16 row sum,
row max, softmax, layer norm; f64 sum) and the same IR shapes in the other
dtype mixes, each checked twice: against a float64 formula of the inputs and
against the IR interpreter (which keeps the IR's per-step roundings).

Against float64 (``tests/parity.py``, the north star's tolerances): f64
outputs 1e-12, f32 outputs 1e-5, f16 outputs 1e-3 (f16 operands, f32
arithmetic, one rounding at the store: ``+ 2^-11 * |ref|``), each relative to
the family's scale -- ``|ref|`` for softmax and rms / l2 norm, ``(|x| +
|mean|) * rstd * |gamma| + |beta|`` for layer norm, ``sum |x|`` for sums and
means, ``|A| @ |v|`` for a dot product; a max over f16 values is exact.

Against the interpreter, the reference spec's own f16 bounds (sum 3e-2,
softmax rtol 3e-2 / atol 3e-3, norms 4e-2; a dot product, whose f16 IR also
rounds every product, atol 0.1): an IR with an f16 accumulator rounds every
fold to f16 (reference ptxc/stmts.py:589-594), which these kernels do not, so
the interpreter of such an IR is itself that far from float64.
"""

from __future__ import annotations

import numpy as np
import pytest

from emmy_ir import synth
from gpu_util import run_on_gpu, shaped
from oracle import formulas as F
from oracle.interp import run_ir
from parity import check as parity_check

pytestmark = pytest.mark.gpu

def _tol(out_dt, kind):
    if out_dt == "f64":
        return 1e-12, 1e-12
    if out_dt == "f32":
        return 1e-5, 1e-5
    # dot: the f16 IR rounds every product and every fold to f16
    return {"sum": (3e-2, 3e-2), "max": (0.0, 0.0), "softmax": (3e-2, 3e-3),
            "norm": (4e-2, 4e-2), "dot": (3e-2, 1e-1)}[kind]


def _check(got, ref, rtol, atol, what):
    got = np.asarray(got, dtype=np.float64).reshape(-1)
    ref = np.asarray(ref, dtype=np.float64).reshape(-1)
    err = np.abs(got - ref)
    bad = err > atol + rtol * np.abs(ref)
    assert not bad.any(), (f"{what}: {int(bad.sum())} of {err.size} outside; worst |d| "
                           f"{float(err.max()):.3g}")


def _run(kop, meta, kind, ref_fn, scale_fn=None):
    plan, host, out = run_on_gpu(kop, meta)
    assert plan["family"] == "rowop", plan["family"]
    x = shaped(meta, host)
    y_name = plan["args"]["y"]
    ydt = meta_dtype(meta, y_name)
    rtol, atol = _tol(ydt, kind)
    ref = np.asarray(ref_fn(x), dtype=np.float64)
    got = np.asarray(out[y_name], dtype=np.float64).reshape(ref.shape)
    x_name = next(a["name"] for a in meta["args"] if not a.get("output") and "data" not in a)
    case = (f"rowop {kind} {kop.name} {meta_dtype(meta, x_name)}->{ydt} "
            f"{list(np.shape(x[x_name]))}")
    if kind == "max":
        npdt = {"f32": np.float32, "f16": np.float16, "f64": np.float64}[ydt]
        assert np.array_equal(got, ref.astype(npdt).astype(np.float64)), case
    else:
        parity_check(got, ref, None if scale_fn is None else scale_fn(x), case=case,
                     family=f"rowop_{kind}", dtype=ydt)
    want = run_ir(kop, meta, host)[y_name]
    _check(out[y_name], want, rtol, atol, "vs interpreter")
    return plan


def _sum_scale(ax, mean=False):
    def fn(x):
        a = np.abs(x["x"].astype(np.float64))
        return a.mean(ax) if mean else a.sum(ax)
    return fn


def _ln_scale(x):
    return F.layernorm_abs_scale(x["x"].astype(np.float64),
                                 None if "gamma" not in x else x["gamma"].astype(np.float64),
                                 None if "beta" not in x else x["beta"].astype(np.float64), 1e-5)


def meta_dtype(meta, name):
    return next(a["dtype"] for a in meta["args"] if a["name"] == name)


@pytest.mark.parametrize("dt,acc", [("f16", "f16"), ("f16", "f32"), ("f64", "f64")])
@pytest.mark.parametrize("op", ["sum", "mean", "max"])
@pytest.mark.parametrize("shape,axis", [([64, 512], -1), ([33, 7], -1), ([96, 40], 0),
                                        ([8, 300, 24], 1), ([4096, 3000], -1)])
def test_reduce(shape, axis, op, dt, acc):
    if acc == "f16" and shape[axis] > 1024:
        pytest.skip("an f16 accumulator over thousands of folds is itself outside the f16 bound")
    kop, meta = synth.retype(*synth.reduce(shape, axis, op, dtype="f32"), dt, acc=acc)
    kind = "max" if op == "max" else "sum"
    ax = axis % len(shape)

    def ref(x):
        v = x["x"].astype(np.float64)
        return {"sum": v.sum(ax), "mean": v.mean(ax), "max": v.max(ax)}[op]
    _run(kop, meta, kind, ref, _sum_scale(ax, op == "mean"))


def test_reduce_f64_whole_tensor():
    kop, meta = synth.retype(*synth.reduce([4096], None, "sum", dtype="f32"), "f64")
    _run(kop, meta, "sum", lambda x: x["x"].astype(np.float64).sum(), _sum_scale(None))


@pytest.mark.parametrize("dt,acc", [("f16", "f16"), ("f16", "f32"), ("f64", "f64")])
@pytest.mark.parametrize("shape,dim", [([64, 512], -1), ([64, 32], -1), ([2, 4, 64, 3000], -1),
                                       ([96, 40], 0), ([300, 4096], -1), ([33, 1024], -1),
                                       ([5, 2048], -1)])
def test_softmax(shape, dim, dt, acc):
    kop, meta = synth.retype(*synth.softmax(shape, dim=dim), dt, acc=acc)
    _run(kop, meta, "softmax",
         lambda x: F.softmax(x["x"].astype(np.float64), axis=dim, out_dtype=np.float64))


@pytest.mark.parametrize("dt,acc", [("f16", "f16"), ("f16", "f32"), ("f64", "f64")])
@pytest.mark.parametrize("rows,cols", [(64, 512), (100, 4096), (7, 96), (33, 1024), (17, 2048)])
def test_layernorm(rows, cols, dt, acc):
    kop, meta = synth.retype(*synth.layernorm(rows, cols), dt, acc=acc)

    def ref(x):
        return F.layernorm(x["x"].astype(np.float64), x["gamma"].astype(np.float64),
                           x["beta"].astype(np.float64), 1e-5, out_dtype=np.float64)
    _run(kop, meta, "norm", ref, _ln_scale)


@pytest.mark.parametrize("dt,acc", [("f16", "f32"), ("f64", "f64")])
def test_rmsnorm_and_l2(dt, acc):
    kop, meta = synth.retype(*synth.rmsnorm(128, 512, eps=1e-5), dt, acc=acc)
    _run(kop, meta, "norm", lambda x: F.rmsnorm(x["x"].astype(np.float64), x["w"].astype(np.float64),
                                                1e-5, out_dtype=np.float64))
    kop, meta = synth.retype(*synth.l2norm(64, 256), dt, acc=acc)
    _run(kop, meta, "norm", lambda x: F.l2norm(x["x"].astype(np.float64), out_dtype=np.float64))


@pytest.mark.parametrize("cols", [1024, 2048, 4096])
def test_rmsnorm_f16_wide_rows(cols):
    """f16 rows held in registers: one warp per row up to 2048, two at 4096."""
    kop, meta = synth.retype(*synth.rmsnorm(37, cols, eps=1e-5), "f16", acc="f32")
    _run(kop, meta, "norm", lambda x: F.rmsnorm(x["x"].astype(np.float64), x["w"].astype(np.float64),
                                                1e-5, out_dtype=np.float64))


@pytest.mark.parametrize("dt", ["f16", "f64"])
def test_norms_without_weights(dt):
    """Null weight / bias / eps pointers: nothing may be loaded through them."""
    kop, meta = synth.retype(*synth.rmsnorm(64, 512, eps=1e-5, weight=False), dt, acc="f32" if dt == "f16" else dt)
    _run(kop, meta, "norm", lambda x: F.rmsnorm(x["x"].astype(np.float64), None, 1e-5,
                                                out_dtype=np.float64))
    kop, meta = synth.retype(*synth.layernorm(64, 512, affine=False), dt)
    _run(kop, meta, "norm", lambda x: F.layernorm(x["x"].astype(np.float64), None, None, 1e-5,
                                                  out_dtype=np.float64), _ln_scale)


@pytest.mark.parametrize("dt", ["f32", "f16"])
def test_dot_with_vector(dt):
    kop, meta = synth.matvec(512, 1000, dtype=dt)
    _run(kop, meta, "dot",
         lambda x: x["A"].astype(np.float64) @ x["v"].astype(np.float64),
         lambda x: np.abs(x["A"].astype(np.float64)) @ np.abs(x["v"].astype(np.float64)))


def test_mixed_output_dtype():
    """f16 rows reduced into an f32 output, f64 rows into f32 (the reference
    spec's f64 sum is checked as f32)."""
    kop, meta = synth.retype(*synth.reduce([64, 512], -1, "sum", dtype="f32"), "f16", acc="f32")
    meta["args"] = [dict(a, dtype="f32") if a["name"] == "y" else a for a in meta["args"]]
    _run(kop, meta, "sum", lambda x: x["x"].astype(np.float64).sum(-1), _sum_scale(-1))
    kop, meta = synth.retype(*synth.reduce([4096], None, "sum", dtype="f32"), "f64")
    meta["args"] = [dict(a, dtype="f32") if a["name"] == "y" else a for a in meta["args"]]
    _run(kop, meta, "sum", lambda x: x["x"].astype(np.float64).sum(), _sum_scale(None))
