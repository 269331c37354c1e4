"""The reference's fixture kernels rebuilt with ``emmy_ir.synth``.

Each entry rebuilds one fixture of the reference's test suite
(``tests/variants/<id>``) as Kernel IR of the same statement shape, the same
argument names, shapes, seeds and literal data, so ``make_inputs`` gives the
very inputs the reference harness fed it and the stored golden output
(``goldens.npz``) is the expected result.  Used by the CPU pin tests (oracle
vs golden) and the GPU parity tests (kernel vs golden), neither of which
needs the reference checkout.
"""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent

_TABLE = None
_ARRAYS = None


def table() -> dict:
    global _TABLE
    if _TABLE is None:
        _TABLE = json.loads((HERE / "goldens.json").read_text())
    return _TABLE


def golden(fid: str):
    """(expected values, positions or None for the whole output, table entry)."""
    global _ARRAYS
    if _ARRAYS is None:
        _ARRAYS = dict(np.load(HERE / "goldens.npz"))
    entry = table()[fid]
    idx = _ARRAYS.get(f"{fid}__index")
    return _ARRAYS[f"{fid}__expected"], idx, entry


def _seeds(fid):
    return {a["name"]: a["seed"] for a in table()[fid]["args"] if "seed" in a}


def _c(name, value):
    return ("const", name, value)


# fixture id -> (expression, dtype); n, shape and the output name come from the table
POINTWISE = {
    "v_p_2d": (("add", _c("add_c1", 3.0), ("multiply", _c("mul_c1", 2.0), "x")), "f32"),
    "v_p_big": (("add", "x0", "x1"), "f32"),
    "v_p_div": (("multiply", "x", ("reciprocal", _c("div_c1", 4.0))), "f32"),
    "v_p_exp": (("exp", "x"), "f32"),
    "v_p_maximum": (("maximum", "x0", "x1"), "f32"),
    "v_p_odd": (("multiply", _c("mul_c1", 3.5), "x"), "f32"),
    "v_p_one": (("multiply", _c("mul_c1", 2.0), "x"), "f32"),
    "v_p_sqrt_abs": (("sqrt", ("abs", "x")), "f32"),
    "v_p_sub": (("subtract", "x0", "x1"), "f32"),
    "v_p_tiny": (("add", "x0", "x1"), "f32"),
    "v_p_where": (("where", ("greater", "x", _c("gt_c1", 0.0)), "x", "y"), "f32"),
    "w_p_f16": (("add", "x0", "x1"), "f16"),
    "w_p_f64": (("multiply", _c("mul_c1", 2.0), "x"), "f64"),
    "w_p_fma": (("add", "x2", ("multiply", "x0", "x1")), "f32"),
    "w_p_neg": (("negative", "x"), "f32"),
    "w_p_pow": (("multiply", "x", "x"), "f32"),
    "w_p_tanh": (("tanh", "x"), "f32"),
}


def build(fid: str):
    """(KernelOp, meta kernel dict) of the replica of fixture ``fid``."""
    from emmy_ir import synth
    entry = table()[fid]
    if fid in POINTWISE:
        expr, dt = POINTWISE[fid]
        shape = entry["shape"]
        n = int(np.prod(shape)) if shape else 1
        return synth.pointwise(n, expr, dt, shape=shape, out=entry["output"], seeds=_seeds(fid),
                               entry=f"k_{entry['output']}_pointwise")
    raise KeyError(f"no replica for {fid!r}")


def replica_ids() -> list:
    return [f for f in sorted(table()) if f in POINTWISE]


def same_inputs(fid: str, meta: dict) -> bool:
    """The replica declares the fixture's arguments (name, dtype, shape, seed / data)."""
    def norm(args):
        return sorted((a["name"], a["dtype"], tuple(a["shape"]), a.get("seed"),
                       tuple(a["data"]) if "data" in a else None, bool(a.get("output")))
                      for a in args)
    return norm(meta["args"]) == norm(table()[fid]["args"])


def compare(fid: str, out: np.ndarray):
    """Max violation of the fixture's tolerance (<= 0 passes) and a message."""
    exp, idx, entry = golden(fid)
    got = np.asarray(out).reshape(-1)
    sel = got if idx is None else got[idx]
    e64 = exp.astype(np.float64)
    g64 = sel.astype(np.float64)
    tol = entry["atol"] + entry["rtol"] * np.abs(e64)
    err = np.abs(g64 - e64)
    bad = np.isnan(g64) != np.isnan(e64)
    worst = float(np.max(np.where(np.isnan(e64), 0.0, err - tol))) if err.size else 0.0
    if bad.any():
        worst = float("inf")
    msg = f"{fid}: max |err| {float(np.nanmax(err)) if err.size else 0.0:.3g}, " \
          f"rtol {entry['rtol']}, atol {entry['atol']}"
    return worst, msg
