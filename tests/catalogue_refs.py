"""float64 references and tolerances for the shape catalogue (``emmy_ir.catalogue``).

Each entry: ``fn(inputs) -> expected output`` over the package's host inputs
(numpy, by argument name, shaped), and the (rtol, atol) the reference checks
that problem with (``tools/specs/*.py``).  Helpers restate the math in float64.
"""

from __future__ import annotations

import math

import numpy as np

from oracle import formulas as F

f64 = lambda a: np.asarray(a, dtype=np.float64)  # noqa: E731
_erf = np.vectorize(math.erf)


def _attn(div):
    def fn(x):
        q = f64(x["q"]).reshape(x["q"].shape[-2:])
        kt = f64(x["k"]).reshape(x["k"].shape[-2:])
        v = f64(x["v"]).reshape(x["v"].shape[-2:])
        return F.softmax(q @ kt / div, axis=-1, out_dtype=np.float64) @ v
    return fn


def _mm(x):
    return np.matmul(f64(x["A"]), f64(x["B"]))


def _red(op, axis):
    def fn(x):
        v = f64(x["x"])
        return {"sum": v.sum(axis), "mean": v.mean(axis), "max": v.max(axis)}[op]
    return fn


def _sm(axis=-1):
    return lambda x: F.softmax(f64(x["x"]), axis=axis, out_dtype=np.float64)


def _rms(x):
    return F.rmsnorm(f64(x["x"]), f64(x["w"]), 1e-5, out_dtype=np.float64)


def _ln(affine):
    def fn(x):
        v = f64(x["x"])
        y = (v - v.mean(-1, keepdims=True)) / np.sqrt(v.var(-1, keepdims=True) + 1e-5)
        return y * f64(x["gamma"]) + f64(x["beta"]) if affine else y
    return fn


def _gelu(v):
    return 0.5 * v * (1.0 + _erf(v / math.sqrt(2.0)))


def _gelu_tanh(v):
    return 0.5 * v * (1.0 + np.tanh(math.sqrt(2.0 / math.pi) * (v + 0.044715 * v ** 3)))


x0 = lambda x: f64(x["x0"])  # noqa: E731

REFS = {
    "adv_layernorm_affine": (_ln(True), 1e-3, 1e-4),
    "adv_mm_gelu": (lambda x: _gelu(_mm(x)), 1e-4, 1e-4),
    "adv_tiny_add": (lambda x: x0(x) + f64(x["x1"]), 0, 0),
    "adv_tiny_sum": (_red("sum", None), 1e-6, 1e-6),
    "adv_red3d_mid": (_red("sum", 1), 1e-3, 1e-4),
    "adv_where_pow": (lambda x: np.where(x0(x) > 0, x0(x) ** 2, -x0(x)), 1e-5, 1e-6),
    "adv_softmax64": (_sm(), 1e-6, 1e-7),
    "adv_attn_noscale": (_attn(1.0), 1e-3, 1e-4),
    "adv_nan_ne": (lambda x: np.ones_like(x0(x)), 0, 0),
    "adv_nan_eq": (lambda x: np.full_like(x0(x), 2.0), 0, 0),
    "adv_mm_bias_relu": (lambda x: np.maximum(_mm(x) + f64(x["bias"]), 0), 1e-4, 1e-4),
    "adv_bmm": (_mm, 1e-4, 1e-4),
    "b_sum_t64": (_red("sum", None), 1e-4, 1e-3),
    "b_sum_t256": (_red("mean", None), 1e-4, 1e-5),
    "b_softmax_1024_t256": (_sm(), 1e-4, 1e-6),
    "b_rms_t256": (_rms, 1e-4, 1e-4),
    "x_p_log": (lambda x: np.log(x0(x) ** 2 + 10.0), 1e-5, 1e-6),
    "x_p_recip": (lambda x: 1.0 / (x0(x) ** 2 + 5.0), 1e-5, 1e-6),
    "x_p_rsqrt": (lambda x: 1.0 / np.sqrt(x0(x) ** 2 + 1.0), 1e-5, 1e-6),
    "x_p_sigmoid": (lambda x: 1.0 / (1.0 + np.exp(-x0(x))), 1e-5, 1e-6),
    "x_p_silu": (lambda x: x0(x) / (1.0 + np.exp(-x0(x))), 1e-5, 1e-6),
    "z_t32_sum": (_red("sum", None), 1e-4, 1e-3),
    "z_t1024_sum": (_red("sum", None), 1e-4, 1e-2),
    "z_prime": (lambda x: x0(x) * 2.5 + 0.5, 1e-6, 1e-6),
    "z_3d_point": (lambda x: x0(x) * 3.0, 1e-6, 1e-6),
    "z_big_point": (lambda x: x0(x) + 1.0, 1e-6, 1e-6),
    "z_red_mid3": (_red("sum", 1), 1e-4, 1e-4),
    "z_red_row1": (_red("sum", -1), 1e-6, 1e-6),
    "z_mean_col": (_red("mean", 0), 1e-5, 1e-5),
    "z_mm_k8": (_mm, 1e-4, 1e-4),
    "z_sm_row1": (_sm(), 1e-6, 1e-6),
    "z_sm_row128": (_sm(), 1e-4, 1e-6),
    "z_rms_col": (_rms, 1e-4, 1e-4),
    "z_sm_4d": (_sm(), 1e-4, 1e-6),
    "z_rowmax32": (_red("max", -1), 0, 0),
    "h_mm_96x80x48": (_mm, 1e-4, 1e-4),
    "h_mm_1024": (_mm, 1e-3, 1e-3),
    "h_mm_64": (_mm, 1e-4, 1e-4),
    "h_mm_128": (_mm, 1e-4, 1e-4),
    "h_bmm": (_mm, 1e-4, 1e-4),
    "ln_512": (_ln(False), 1e-3, 1e-4),
    "ln_1024": (_ln(False), 1e-3, 1e-4),
    "op_gelu": (lambda x: _gelu(3.0 * x0(x)), 1e-5, 1e-5),
    "op_gelu_tanh": (lambda x: _gelu_tanh(3.0 * x0(x)), 1e-5, 1e-5),
    "op_gelu16": (lambda x: _gelu(3.0 * x0(x)), 1e-2, 1e-2),
    "op_softplus": (lambda x: np.log1p(np.exp(3.0 * x0(x))), 1e-5, 1e-5),
    "op_cos_sin": (lambda x: np.cos(4.0 * x0(x)) + np.sin(4.0 * f64(x["x1"])), 1e-5, 1e-5),
    "op_erf64": (lambda x: _erf(2.0 * x0(x)), 1e-12, 1e-13),
    "s_sum_1m": (_red("sum", None), 1e-4, 1e-2),
    "s_sumdim0": (_red("sum", 0), 1e-4, 1e-4),
    "s_mean_rows": (_red("mean", -1), 1e-4, 1e-5),
    "s_mm_2048": (_mm, 1e-3, 1e-3),
    "s_mm_splitk": (_mm, 1e-3, 1e-3),
    "s_softmax_big": (_sm(), 1e-4, 1e-7),
    "dt_rowsum16": (_red("sum", -1), 3e-2, 3e-2),
    "dt_rowmax16": (_red("max", -1), 2e-2, 2e-2),
    "dt_softmax16": (_sm(), 3e-2, 3e-3),
    "dt_layernorm16": (_ln(False), 4e-2, 4e-2),
    "dt_sum64": (_red("sum", None), 1e-5, 1e-5),
    "dt_add64": (lambda x: x0(x) + f64(x["x1"]), 1e-10, 1e-12),
    "dt_exp64": (lambda x: np.exp(3.0 * x0(x)), 1e-14, 1e-14),
    "dt_log64": (lambda x: np.log(np.abs(x0(x)) + 0.5), 1e-12, 1e-13),
    "dt_pow64": (lambda x: np.power(np.abs(x0(x)) + 0.5, 1.7), 1e-12, 1e-13),
    "dt_tanh64": (lambda x: np.tanh(2.0 * x0(x)), 1e-14, 1e-15),
    "dt_mul16_64": (lambda x: x0(x) * f64(x["x1"]), 2e-2, 2e-2),
    "h16_add4k": (lambda x: x0(x) + f64(x["x1"]), 1e-2, 1e-2),
    "h16_exp": (lambda x: np.exp(x0(x)), 1e-2, 1e-2),
    "n_row32_sum": (_red("sum", -1), 1e-4, 1e-4),
    "n_row32_mean": (_red("mean", -1), 1e-4, 1e-4),
    "n_softmax32": (_sm(), 1e-3, 1e-5),
    "n_row7": (_red("sum", -1), 1e-4, 1e-4),
}
for _id, _s, _d in (("x_attn_s48_h96", 48, 9.797959), ("x_attn_s100_h32", 100, 5.656854),
                    ("x_attn_s33_h64", 33, 8.0), ("x_attn_s128_h96", 128, 9.797959),
                    ("x_attn_s64_h48", 64, 6.928203), ("e_attn_s32_h32", 32, 5.656854),
                    ("e_attn_s64_h256", 64, 16.0), ("e_attn_s512_h16", 512, 4.0),
                    ("e_attn_s16_h64", 16, 8.0), ("e_attn_s256_h16", 256, 4.0),
                    ("g_attn_s128_h64", 128, 8.0), ("g_attn_s256_h32", 256, 5.656854),
                    ("g_attn_s128_h128", 128, 11.313708), ("g_attn_s64_h128", 64, 11.313708),
                    ("g_attn_s256_h64", 256, 8.0), ("z_attn_h16", 64, 4.0),
                    ("h_attn_48x16", 48, 4.0), ("h_attn_96x32", 96, 5.656854),
                    ("s_attn_big", 256, 11.313708)):
    REFS[_id] = (_attn(_d), 1e-3, 1e-4)


def host_inputs(pairs) -> dict:
    """Seeded inputs for every argument a package's caller provides."""
    from oracle.interp import make_inputs
    host = {}
    for _, meta in pairs:
        for k, v in make_inputs(meta).items():
            a = next(x for x in meta["args"] if x["name"] == k)
            if not a.get("output") and not a.get("intermediate"):
                host[k] = v
    return host


def shaped(pairs, host) -> dict:
    shapes = {a["name"]: tuple(a["shape"]) for _, m in pairs for a in m["args"]}
    return {k: v.reshape(shapes[k]) if shapes[k] else v for k, v in host.items()}


def final_output(pairs) -> str:
    meta = pairs[-1][1]
    return next(a["name"] for a in meta["args"] if a.get("output"))


def check(got, want, rtol, atol, what):
    got = np.asarray(got, dtype=np.float64).reshape(-1)
    want = np.asarray(want, dtype=np.float64).reshape(-1)
    assert got.shape == want.shape, (what, got.shape, want.shape)
    err = np.abs(got - want)
    bad = ~(err <= atol + rtol * np.abs(want))
    assert not bad.any(), (f"{what}: {int(bad.sum())} of {err.size} outside rtol {rtol} atol {atol}; "
                           f"worst |d| {float(np.nanmax(err)):.3g}")
