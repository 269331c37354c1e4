"""A catalogue of problem shapes as synthesised Kernel IR packages.

The reference generates its problem packages from torch snippets with the
emmy generator (``tools/specs/*.py`` lists them; ``tools/generate_corpus.sh``
drives the generator).  The generator is not available here, so this module
restates each catalogued shape -- sizes, dtypes, the op chain, the constants --
with the synthesiser in ``emmy_ir.synth``, in the IR shapes of the reference
fixtures.  ``build(id)`` returns the package's kernels as
``[(KernelOp, meta kernel entry), ...]`` (two for a matmul followed by an
elementwise kernel); ``write(id, dir)`` writes the package as IR JSON.

``SKIPPED`` names the shapes the synthesiser cannot express, with the reason.
"""

from __future__ import annotations

import math

from . import synth


def _pw(n, expr, dtype="f32", shape=None, **kw):
    return [synth.pointwise(n, expr, dtype, shape=shape, **kw)]


def _attn(S, D, div):
    return [synth.attention(1, 1, S, D, dtype="f32", scale_div=div, k_transposed=True)]


def _mm(M, N, K, batch=1, **kw):
    tm = math.gcd(M, 64)
    tn = math.gcd(N, 64)
    rm = math.gcd(tm, 4)
    rn = math.gcd(tn, 4)
    bk = kw.pop("bk", math.gcd(K, 16))
    return [synth.matmul(M, N, K, batch=batch, tm=tm, tn=tn, rm=rm, rn=rn, bk=bk, **kw)]


def _mm_then(M, N, K, expr):
    """A matmul writing ``mm``, then an elementwise kernel of ``mm``."""
    k1, m1 = synth.matmul(M, N, K, tm=math.gcd(M, 64), tn=math.gcd(N, 64), rm=4, rn=4,
                          bk=math.gcd(K, 16), entry="k_mm__partial", c_name="mm")
    m1["final"] = False
    k2, m2 = synth.pointwise(M * N, expr, "f32", shape=[M, N], entry="k_mm")
    for a in m2["args"]:
        if a["name"] == "mm":
            a["intermediate"] = True
            a.pop("seed", None)
    return [(k1, m1), (k2, m2)]


def _typed(pair, dtype, acc=None, out=None):
    kop, meta = synth.retype(*pair, dtype, acc=acc)
    if out:
        meta["args"] = [dict(a, dtype=out) if a.get("output") else a for a in meta["args"]]
    return [(kop, meta)]


def _ln(rows, cols, affine):
    return [synth.layernorm(rows, cols, affine=affine)]


X = "x0"
SPECS = {
    # adversarial shapes
    "adv_layernorm_affine": lambda: _ln(64, 512, True),
    "adv_mm_gelu": lambda: _mm_then(64, 64, 64, ("gelu", "mm")),
    "adv_tiny_add": lambda: _pw(3, ("add", "x0", "x1")),
    "adv_tiny_sum": lambda: [synth.reduce([4], None, "sum")],
    "adv_red3d_mid": lambda: [synth.reduce([4, 128, 64], 1, "sum")],
    "adv_where_pow": lambda: _pw(4096, ("where", ("greater", X, ("imm", 0.0)),
                                        ("pow", X, ("imm", 2.0)), ("negative", X))),
    "adv_softmax64": lambda: _typed(synth.softmax([64, 256]), "f64"),
    "adv_attn_noscale": lambda: _attn(32, 64, 1.0),
    "adv_nan_ne": lambda: _pw(1024, ("where", ("not_equal", X, ("imm", float("nan"))),
                                     ("imm", 1.0), ("imm", 2.0))),
    "adv_nan_eq": lambda: _pw(1024, ("where", ("equal", X, ("imm", float("nan"))),
                                     ("imm", 1.0), ("imm", 2.0))),
    "adv_mm_bias_relu": lambda: synth.mm_bias_relu_chain(64, 64, 64, tm=64, tn=64, rm=4, rn=4),
    "adv_bmm": lambda: _mm(8, 8, 16, batch=4, bk=4),
    # attention, one (batch, head), f32, k pre-transposed
    "x_attn_s48_h96": lambda: _attn(48, 96, 9.797959),
    "x_attn_s100_h32": lambda: _attn(100, 32, 5.656854),
    "x_attn_s33_h64": lambda: _attn(33, 64, 8.0),
    "x_attn_s128_h96": lambda: _attn(128, 96, 9.797959),
    "x_attn_s64_h48": lambda: _attn(64, 48, 6.928203),
    "e_attn_s32_h32": lambda: _attn(32, 32, 5.656854),
    "e_attn_s64_h256": lambda: _attn(64, 256, 16.0),
    "e_attn_s512_h16": lambda: _attn(512, 16, 4.0),
    "e_attn_s16_h64": lambda: _attn(16, 64, 8.0),
    "e_attn_s256_h16": lambda: _attn(256, 16, 4.0),
    "g_attn_s128_h64": lambda: _attn(128, 64, 8.0),
    "g_attn_s256_h32": lambda: _attn(256, 32, 5.656854),
    "g_attn_s128_h128": lambda: _attn(128, 128, 11.313708),
    "g_attn_s64_h128": lambda: _attn(64, 128, 11.313708),
    "g_attn_s256_h64": lambda: _attn(256, 64, 8.0),
    "z_attn_h16": lambda: _attn(64, 16, 4.0),
    "h_attn_48x16": lambda: _attn(48, 16, 4.0),
    "h_attn_96x32": lambda: _attn(96, 32, 5.656854),
    "s_attn_big": lambda: _attn(256, 128, 11.313708),
    # block-level reductions and row families
    "b_sum_t64": lambda: [synth.reduce([32768], None, "sum")],
    "b_sum_t256": lambda: [synth.reduce([65536], None, "mean")],
    "b_softmax_1024_t256": lambda: [synth.softmax([64, 1024])],
    "b_rms_t256": lambda: [synth.rmsnorm(64, 2048, eps=1e-5)],
    # elementwise chains
    "x_p_log": lambda: _pw(512, ("log", ("add", ("multiply", X, X), ("imm", 10.0)))),
    "x_p_recip": lambda: _pw(1024, ("reciprocal", ("add", ("multiply", X, X), ("imm", 5.0)))),
    "x_p_rsqrt": lambda: _pw(1024, ("rsqrt", ("add", ("multiply", X, X), ("imm", 1.0)))),
    "x_p_sigmoid": lambda: _pw(1024, ("sigmoid", X)),
    "x_p_silu": lambda: _pw(1024, ("multiply", X, ("sigmoid", X))),
    # fuzzed shapes
    "z_t32_sum": lambda: [synth.reduce([4096], None, "sum")],
    "z_t1024_sum": lambda: [synth.reduce([262144], None, "sum")],
    "z_prime": lambda: _pw(1009, ("add", ("multiply", X, ("imm", 2.5)), ("imm", 0.5))),
    "z_3d_point": lambda: _pw(4 * 8 * 32, ("multiply", X, ("imm", 3.0)), shape=[4, 8, 32]),
    "z_big_point": lambda: _pw(262144, ("add", X, ("imm", 1.0))),
    "z_red_mid3": lambda: [synth.reduce([8, 30, 64], 1, "sum")],
    "z_red_row1": lambda: [synth.reduce([256, 1], -1, "sum")],
    "z_mean_col": lambda: [synth.reduce([32, 128], 0, "mean")],
    "z_mm_k8": lambda: _mm(64, 64, 8, bk=8),
    "z_sm_row1": lambda: [synth.softmax([64, 1])],
    "z_sm_row128": lambda: [synth.softmax([128, 128])],
    "z_rms_col": lambda: [synth.rmsnorm(32, 512, eps=1e-5)],
    "z_sm_4d": lambda: [synth.softmax([2, 3, 16, 256])],
    "z_rowmax32": lambda: [synth.reduce([64, 512], -1, "max")],
    # held-out matmuls
    "h_mm_96x80x48": lambda: _mm(96, 48, 80),
    "h_mm_1024": lambda: _mm(1024, 1024, 1024),
    "h_mm_64": lambda: _mm(64, 64, 64),
    "h_mm_128": lambda: _mm(128, 128, 128),
    "h_bmm": lambda: _mm(32, 32, 64, batch=4),
    # layer norm without affine
    "ln_512": lambda: _ln(64, 512, False),
    "ln_1024": lambda: _ln(32, 1024, False),
    # transcendental elementwise ops
    "op_gelu": lambda: _pw(4096, ("gelu", ("multiply", X, ("imm", 3.0)))),
    "op_gelu_tanh": lambda: _pw(4096, ("gelu_tanh", ("multiply", X, ("imm", 3.0)))),
    "op_gelu16": lambda: _pw(4096, ("gelu", ("multiply", X, ("imm", 3.0))), "f16"),
    "op_softplus": lambda: _pw(4096, ("softplus", ("multiply", X, ("imm", 3.0)))),
    "op_cos_sin": lambda: _pw(2048, ("add", ("cos", ("multiply", "x0", ("imm", 4.0))),
                                     ("sin", ("multiply", "x1", ("imm", 4.0))))),
    "op_erf64": lambda: _pw(2048, ("erf", ("multiply", X, ("imm", 2.0))), "f64"),
    # stress sizes
    "s_sum_1m": lambda: [synth.reduce([1000000], None, "sum")],
    "s_sumdim0": lambda: [synth.reduce([128, 512], 0, "sum")],
    "s_mean_rows": lambda: [synth.reduce([512, 4096], -1, "mean")],
    "s_mm_2048": lambda: _mm(2048, 2048, 2048),
    "s_mm_splitk": lambda: _mm(512, 512, 4096, splits=8),
    "s_softmax_big": lambda: [synth.softmax([64, 4096])],
    # dtype edges
    "dt_rowsum16": lambda: _typed(synth.reduce([64, 512], -1, "sum"), "f16"),
    "dt_rowmax16": lambda: _typed(synth.reduce([64, 512], -1, "max"), "f16"),
    "dt_softmax16": lambda: _typed(synth.softmax([64, 512]), "f16"),
    "dt_layernorm16": lambda: _typed(synth.layernorm(64, 512, affine=False), "f16"),
    "dt_sum64": lambda: _typed(synth.reduce([4096], None, "sum"), "f64", out="f32"),
    "dt_add64": lambda: _pw(2048, ("add", "x0", "x1"), "f64"),
    "dt_exp64": lambda: _pw(2048, ("exp", ("multiply", X, ("imm", 3.0))), "f64"),
    "dt_log64": lambda: _pw(2048, ("log", ("add", ("abs", X), ("imm", 0.5))), "f64"),
    "dt_pow64": lambda: _pw(1024, ("pow", ("add", ("abs", X), ("imm", 0.5)), ("imm", 1.7)), "f64"),
    "dt_tanh64": lambda: _pw(2048, ("tanh", ("multiply", X, ("imm", 2.0))), "f64"),
    "dt_mul16_64": lambda: _pw(2048, ("multiply", "x0", "x1"), "f64", dtypes={"x0": "f16"},
                               out_dtype="f16"),
    "h16_add4k": lambda: _pw(4096, ("add", "x0", "x1"), "f16"),
    "h16_exp": lambda: _pw(2048, ("exp", X), "f16"),
    # small rows
    "n_row32_sum": lambda: [synth.reduce([64, 32], -1, "sum")],
    "n_row32_mean": lambda: [synth.reduce([64, 32], -1, "mean")],
    "n_softmax32": lambda: [synth.softmax([64, 32])],
    "n_row7": lambda: [synth.reduce([33, 7], -1, "sum")],
}

SKIPPED = {
    "z_mm_k17": "K = 17 is not a multiple of a 16-byte cp.async copy; the reference's IR for it "
                "(guarded staging) comes from the generator, which is not available",
    "z_mm_n1": "N = 1 is narrower than one 16-byte copy of B (same reason)",
    "h_mm_odd": "97 x 83 x 59 needs guarded tiles in the IR (same reason)",
}


def ids() -> list:
    return sorted(SPECS)


def build(spec_id: str) -> list:
    """``[(KernelOp, meta kernel entry), ...]`` of the package, in launch order."""
    return SPECS[spec_id]()


def write(spec_id: str, directory) -> list:
    """Write the package (IR JSON per kernel + meta.json); returns the IR paths."""
    from .serialize import write_chain
    return write_chain(directory, build(spec_id), {"id": spec_id})
