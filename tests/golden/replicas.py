"""The reference's fixture kernels rebuilt with ``emmy_ir.synth``.

Each entry rebuilds one fixture of the reference's test suite
(``tests/variants/<id>``) as Kernel IR of the same statement shape, with a map
from the replica's argument names to the fixture's; the inputs are built from
the fixture's own argument table (seeds, literal data) exactly as the
reference harness builds them, so the stored golden output (``goldens.npz``)
is the expected result.  Used by the CPU pin tests (oracle
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


def _rows(fid):
    e = table()[fid]
    return {a["name"]: a for a in e["args"]}


# fixture id -> (builder of the replica, {replica argument: fixture argument})
def _other_replicas():
    from emmy_ir import synth
    R = {}
    for fid, rows, cols in (("v_f_rms_512", 128, 512), ("w_f_rms_2048", 16, 2048)):
        R[fid] = (lambda rows=rows, cols=cols: synth.rmsnorm(rows, cols, eps=1e-5),
                  {"y": "mul_1"})
    R["v_f_l2_256"] = (lambda: synth.l2norm(128, 256), {"y": "div"})
    for fid, shape, dim in (("v_f_softmax_1024", [32, 1024], -1), ("v_f_softmax_384", [128, 384], -1),
                            ("w_f_softmax_2048", [16, 2048], -1), ("w_f_softmax_dim0", [128, 64], 0)):
        R[fid] = (lambda shape=shape, dim=dim: synth.softmax(shape, dim=dim), {"y": "softmax"})
    for fid, shape, axis, op in (("v_r_100000", [100000], -1, "sum"), ("v_r_3d", [8, 32, 256], -1, "sum"),
                                 ("v_r_4096", [4096], -1, "sum"), ("v_r_row_1000", [96, 1000], -1, "mean"),
                                 ("v_r_row_300", [48, 300], -1, "sum"), ("v_r_t256", [65536], -1, "sum"),
                                 ("w_r_dim0", [64, 128], 0, "sum"), ("w_r_mid", [8, 64, 32], 1, "sum"),
                                 ("w_r_odd_row", [17, 777], -1, "sum"), ("w_r_t512", [131072], -1, "sum")):
        out = table()[fid]["output"]
        names = {"y": out, "mean_count": "mean_keepdim_count"}
        R[fid] = (lambda shape=shape, axis=axis, op=op: synth.reduce(shape, axis, op), names)
    for fid, M, N, K, batch in (("v_m_256", 256, 256, 256, 1), ("v_m_rect_small", 64, 32, 128, 1),
                                ("v_m_tall", 512, 64, 128, 1), ("v_m_wide", 128, 512, 64, 1),
                                ("w_m_1024", 1024, 128, 128, 1), ("w_m_batch", 64, 64, 64, 4),
                                ("w_m_k96", 128, 64, 96, 1)):
        R[fid] = (lambda M=M, N=N, K=K, batch=batch: synth.matmul(M, N, K, batch=batch, tm=32, tn=32),
                  {"A": "x0", "B": "x1", "C": "matmul"})
    for fid, S, D, Dv in (("v_a_128", 128, 128, 128), ("v_a_32x256", 32, 256, 32),
                          ("v_a_64x128", 64, 128, 64), ("w_a_256", 256, 64, 64),
                          ("w_a_head64", 128, 64, 64)):
        div = _rows(fid)["div_c1"]["data"][0]
        R[fid] = (lambda S=S, D=D, Dv=Dv, div=div: synth.attention(
            1, 1, S, D, dtype="f32", scale_div=div, k_transposed=True, Dv=Dv),
            {"k": "kt", "o": "matmul_1"})
    return R


_OTHERS = None


def _others():
    global _OTHERS
    if _OTHERS is None:
        _OTHERS = _other_replicas()
    return _OTHERS


def build(fid: str):
    """(KernelOp, meta kernel dict, {replica argument: fixture argument}) of fixture ``fid``'s replica."""
    from emmy_ir import synth
    entry = table()[fid]
    if fid in POINTWISE:
        expr, dt = POINTWISE[fid]
        shape = entry["shape"]
        n = int(np.prod(shape)) if shape else 1
        kop, meta = synth.pointwise(n, expr, dt, shape=shape, out=entry["output"],
                                    seeds=_seeds(fid), entry=f"k_{entry['output']}_pointwise")
        return kop, meta, {a["name"]: a["name"] for a in meta["args"]}
    if fid in _others():
        make, names = _others()[fid]
        kop, meta = make()
        return kop, meta, {a["name"]: names.get(a["name"], a["name"]) for a in meta["args"]}
    raise KeyError(f"no replica for {fid!r}")


def replica_ids() -> list:
    return [f for f in sorted(table()) if f in POINTWISE or f in _others()]


def fixture_inputs(fid: str, meta: dict, names: dict) -> dict:
    """The reference harness's seeded inputs, keyed by the replica's argument names."""
    from oracle.interp import make_inputs
    host = make_inputs({"args": table()[fid]["args"]})
    return {mine: host[theirs] for mine, theirs in names.items()}


def same_inputs(fid: str, meta: dict, names: dict) -> bool:
    """Every replica argument maps to a fixture argument of the same dtype and size,
    and the fixture's literal constants equal the replica's."""
    theirs = _rows(fid)
    if sorted(names.values()) != sorted(theirs):
        return False
    for a in meta["args"]:
        t = theirs[names[a["name"]]]
        n_mine = int(np.prod(a["shape"])) if a["shape"] else 1
        n_theirs = int(np.prod(t["shape"])) if t["shape"] else 1
        if a["dtype"] != t["dtype"] or n_mine != n_theirs or bool(a.get("output")) != bool(t.get("output")):
            return False
        if ("data" in a) != ("data" in t):
            return False
        if "data" in a and not np.array_equal(np.asarray(a["data"], np.float64),
                                              np.asarray(t["data"], np.float64)):
            return False
    return True


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
