"""The oracle is pinned to the reference's golden vectors.

* ``oracle.formulas`` (float64 closed forms cast to f32) reproduces the
  reference ``expected.npz`` files bit for bit.  Scalar constants enter as
  the float64 values meta.json spells (``data``), as the goldens were made.
* ``oracle.interp`` (statement-by-statement evaluation of the IR) matches every
  golden within the fixture's own ``rtol``/``atol``.
* The oracle's input builder reproduces the reference harness
  (``tools/localrun.py:111-118``) and agrees with the product-side builder.
"""

from __future__ import annotations

import numpy as np
import pytest

from conftest import load_variant, needs_reference, reference_variants
from oracle import formulas as F
from oracle.interp import make_inputs, run_ir

FORMULA = {
    "v_f_rms_512": lambda x: F.rmsnorm(x["x"], x["w"], 1e-5),
    "w_f_rms_2048": lambda x: F.rmsnorm(x["x"], x["w"], 1e-5),
    "v_f_l2_256": lambda x: F.l2norm(x["x"]),
    "v_f_softmax_384": lambda x: F.softmax(x["x"]),
    "v_f_softmax_1024": lambda x: F.softmax(x["x"]),
    "w_f_softmax_2048": lambda x: F.softmax(x["x"]),
    "w_f_softmax_dim0": lambda x: F.softmax(x["x"], axis=0),
    "v_r_100000": lambda x: F.reduce(x["x"], None, "sum"),
    "v_r_4096": lambda x: F.reduce(x["x"], None, "sum"),
    "v_r_t256": lambda x: F.reduce(x["x"], None, "sum"),
    "w_r_t512": lambda x: F.reduce(x["x"], None, "sum"),
    "v_r_3d": lambda x: F.reduce(x["x"], -1, "sum"),
    "v_r_row_1000": lambda x: F.reduce(x["x"], -1, "mean"),
    "v_r_row_300": lambda x: F.reduce(x["x"], -1, "sum"),
    "w_r_odd_row": lambda x: F.reduce(x["x"], -1, "sum"),
    "w_r_dim0": lambda x: F.reduce(x["x"], 0, "sum"),
    "w_r_mid": lambda x: F.reduce(x["x"], 1, "sum"),
    "v_m_256": lambda x: F.matmul(x["x0"], x["x1"]),
    "v_m_rect_small": lambda x: F.matmul(x["x0"], x["x1"]),
    "v_m_tall": lambda x: F.matmul(x["x0"], x["x1"]),
    "v_m_wide": lambda x: F.matmul(x["x0"], x["x1"]),
    "w_m_1024": lambda x: F.matmul(x["x0"], x["x1"]),
    "w_m_k96": lambda x: F.matmul(x["x0"], x["x1"]),
    "w_m_batch": lambda x: F.matmul(x["x0"], x["x1"]),
    "v_a_128": lambda x: F.attention(x["q"], x["kt"], x["v"], x["div_c1@data"]),
    "v_a_32x256": lambda x: F.attention(x["q"], x["kt"], x["v"], x["div_c1@data"]),
    "v_a_64x128": lambda x: F.attention(x["q"], x["kt"], x["v"], x["div_c1@data"]),
    "w_a_256": lambda x: F.attention(x["q"], x["kt"], x["v"], x["div_c1@data"]),
    "w_a_head64": lambda x: F.attention(x["q"], x["kt"], x["v"], x["div_c1@data"]),
}
# statement-level interpretation of the attention fixtures with 128+ keys
# takes tens of seconds on CPU; they run under -m slow
SLOW_INTERP = {"v_a_128", "w_a_256"}


def _shaped(meta_kernel, arrays):
    shp = {a["name"]: a["shape"] for a in meta_kernel["args"]}
    return {k: v.reshape(shp[k]) for k, v in arrays.items()}


@needs_reference
@pytest.mark.parametrize("name", sorted(FORMULA))
def test_formula_reproduces_golden(name):
    from conftest import REFERENCE_VARIANTS
    path = REFERENCE_VARIANTS / name
    _, meta, _ = load_variant(path)
    k = meta["kernels"][0]
    x = _shaped(k, make_inputs(k))
    for a in k["args"]:
        if "data" in a and len(a["data"]) == 1:
            x[a["name"] + "@data"] = float(a["data"][0])
    exp = np.load(path / "expected.npz")
    want = exp[exp.files[0]]
    got = FORMULA[name](x).reshape(want.shape)
    assert np.array_equal(got, want)


def _interp_cases():
    out = []
    for p in reference_variants():
        marks = [pytest.mark.slow] if p.name in SLOW_INTERP else []
        out.append(pytest.param(p.name, marks=marks))
    return out


@needs_reference
@pytest.mark.parametrize("name", _interp_cases())
def test_interpreter_matches_golden(name):
    from conftest import REFERENCE_VARIANTS
    path = REFERENCE_VARIANTS / name
    kop, meta, _ = load_variant(path)
    k = meta["kernels"][0]
    out = run_ir(kop, k, make_inputs(k))
    exp = np.load(path / "expected.npz")
    for key in exp.files:
        got = out[key].reshape(exp[key].shape).astype(np.float64)
        assert np.allclose(got, exp[key].astype(np.float64), rtol=meta["rtol"], atol=meta["atol"]), key


def test_input_builders_agree():
    from emmy_ir import synth
    from oracle.interp import make_inputs as oracle_inputs
    _, m = synth.rmsnorm(4, 64)
    a, b = oracle_inputs(m), synth.make_inputs(m)
    for k in a:
        assert np.array_equal(a[k], b[k])
    # localrun: default_rng(seed).standard_normal(n).astype(dtype)
    assert np.array_equal(a["x"], np.random.default_rng(0).standard_normal(256).astype(np.float32))
