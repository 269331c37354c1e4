"""Family matcher: every reference reduction-shaped fixture maps to the right
kernel family and view; synthesised benchmark IR does too; altered IR is
refused (no guessing, no fallback)."""

from __future__ import annotations

import dataclasses

import pytest

from conftest import REFERENCE_VARIANTS, load_variant, needs_reference
from emmy_ir import synth
from emmy_ir.nodes import Assign, ElementwiseImpl
from ptxc import CompileError, Lowerer

EXPECT = {
    "v_f_rms_512": ("rownorm", {"outer": 128, "n": 512, "inner": 1}, {"mode": "rms"}),
    "w_f_rms_2048": ("rownorm", {"outer": 16, "n": 2048, "inner": 1}, {"mode": "rms"}),
    "v_f_l2_256": ("rownorm", {"outer": 128, "n": 256, "inner": 1}, {"mode": "l2"}),
    "v_f_softmax_384": ("softmax", {"outer": 128, "n": 384, "inner": 1}, {}),
    "v_f_softmax_1024": ("softmax", {"outer": 32, "n": 1024, "inner": 1}, {}),
    "w_f_softmax_2048": ("softmax", {"outer": 16, "n": 2048, "inner": 1}, {}),
    "w_f_softmax_dim0": ("softmax", {"outer": 1, "n": 128, "inner": 64}, {}),
    "v_r_100000": ("reduce", {"outer": 1, "n": 100000, "inner": 1}, {"op": "sum", "mean": False}),
    "v_r_3d": ("reduce", {"outer": 256, "n": 256, "inner": 1}, {"op": "sum"}),
    "v_r_4096": ("reduce", {"outer": 1, "n": 4096, "inner": 1}, {"op": "sum"}),
    "v_r_row_1000": ("reduce", {"outer": 96, "n": 1000, "inner": 1}, {"op": "sum", "mean": True}),
    "v_r_row_300": ("reduce", {"outer": 48, "n": 300, "inner": 1}, {"op": "sum"}),
    "v_r_t256": ("reduce", {"outer": 1, "n": 65536, "inner": 1}, {"op": "sum"}),
    "w_r_dim0": ("reduce", {"outer": 1, "n": 64, "inner": 128}, {"op": "sum"}),
    "w_r_mid": ("reduce", {"outer": 8, "n": 64, "inner": 32}, {"op": "sum"}),
    "w_r_odd_row": ("reduce", {"outer": 17, "n": 777, "inner": 1}, {"op": "sum"}),
    "w_r_t512": ("reduce", {"outer": 1, "n": 131072, "inner": 1}, {"op": "sum"}),
}


@needs_reference
@pytest.mark.parametrize("name", sorted(EXPECT))
def test_reference_fixture_maps_to_family(name):
    kop, meta, _ = load_variant(REFERENCE_VARIANTS / name)
    plan = Lowerer(kop, meta["kernels"][0]).plan()
    fam, view, params = EXPECT[name]
    assert plan["family"] == fam
    assert plan["view"] == view
    for k, v in params.items():
        assert plan["params"][k] == v


@needs_reference
def test_rmsnorm_fixture_scalars_are_bound_by_role():
    kop, meta, _ = load_variant(REFERENCE_VARIANTS / "v_f_rms_512")
    plan = Lowerer(kop, meta["kernels"][0]).plan()
    assert plan["args"] == {"x": "x", "y": "mul_1", "w": "w", "eps": "add_c1", "count": "mean_count"}


@needs_reference
@pytest.mark.parametrize("fixture,synth_call", [
    ("v_f_rms_512", lambda: synth.rmsnorm(128, 512, eps=1e-5)),
    ("v_f_softmax_1024", lambda: synth.softmax([32, 1024])),
    ("w_f_softmax_dim0", lambda: synth.softmax([128, 64], dim=0)),
    ("v_f_l2_256", lambda: synth.l2norm(128, 256)),
    ("w_r_mid", lambda: synth.reduce([8, 64, 32], 1, "sum")),
    ("v_r_row_1000", lambda: synth.reduce([96, 1000], -1, "mean")),
])
def test_synthesised_ir_is_the_fixture_shape(fixture, synth_call):
    """The synthesiser writes the same statements as the fixture (up to names)."""
    kop, meta, _ = load_variant(REFERENCE_VARIANTS / fixture)
    skop, smeta = synth_call()
    p_ref = Lowerer(kop, meta["kernels"][0]).plan()
    p_syn = Lowerer(skop, smeta).plan()
    for key in ("family", "view", "params", "symbol"):
        assert p_ref[key] == p_syn[key]
    assert meta["kernels"][0]["grid"] == smeta["grid"]
    assert meta["kernels"][0]["block"] == smeta["block"]
    ref_kinds = [type(s).__name__ for s in kop.body[0].body]
    syn_kinds = [type(s).__name__ for s in skop.body[0].body]
    assert ref_kinds == syn_kinds


@pytest.mark.parametrize("make,family", [
    (lambda: synth.rmsnorm(4096, 512, eps=1e-6), "rownorm"),
    (lambda: synth.softmax([32, 16, 512, 512]), "softmax"),
    (lambda: synth.layernorm(16384, 1024), "rownorm"),
    (lambda: synth.matvec(16384, 16384), "matvec"),
    (lambda: synth.reduce([7, 9, 33], 0, "max"), "reduce"),
])
def test_benchmark_ir_matches(make, family):
    kop, meta = make()
    assert Lowerer(kop, meta).plan()["family"] == family


def _swap_op(kop, name, new_op):
    def fix(st):
        if isinstance(st, Assign) and st.name == name:
            return dataclasses.replace(st, op=ElementwiseImpl(new_op))
        kw = {}
        for attr in ("body", "else_body", "combine_states"):
            if hasattr(st, attr):
                kw[attr] = tuple(fix(s) for s in getattr(st, attr))
        return dataclasses.replace(st, **kw) if kw else st
    return dataclasses.replace(kop, body=tuple(fix(s) for s in kop.body))


@pytest.mark.parametrize("assign,op", [
    ("v4", "rsqrt"),        # sqrt -> rsqrt changes the formula
    ("v5", "copy"),         # drops the reciprocal
    ("v1", "add"),          # x + x instead of x * x
])
def test_altered_rmsnorm_is_refused(assign, op):
    kop, meta = synth.rmsnorm(16, 256)
    with pytest.raises(CompileError, match="no B200 kernel family"):
        Lowerer(_swap_op(kop, assign, op), meta).plan()


def test_altered_combine_is_refused():
    kop, meta = synth.softmax([8, 256])
    # the warp combine's sum of rescaled partials becomes a max
    bad = _swap_op(kop, "acc1", "maximum")
    with pytest.raises(CompileError):
        Lowerer(bad, meta).plan()


def test_partial_block_collective_is_refused():
    kop, meta = synth.softmax([8, 256])
    meta = dict(meta)
    meta["grid"] = [9, 1, 1]   # 9 blocks for 8 rows is fine (extra block idle)
    Lowerer(kop, meta).plan()
    meta["grid"] = [7, 1, 1]   # fewer blocks than rows: part of the Tile never runs
    with pytest.raises(CompileError, match="covers only part"):
        Lowerer(kop, meta).plan()


def test_non_f32_row_families_take_the_typed_kernel():
    kop, meta = synth.reduce([4, 64], -1, "sum", dtype="f64")
    plan = Lowerer(kop, meta).plan()
    assert plan["family"] == "rowop" and plan["params"]["compute"] == "f64"


def test_unsupported_dtype_is_refused_not_guessed():
    kop, meta = synth.reduce([4, 64], -1, "sum", dtype="f32")
    meta["args"] = [dict(a, dtype="i32") if a["name"] == "x" else a for a in meta["args"]]
    with pytest.raises(CompileError, match="f16 / f32 / f64"):
        Lowerer(kop, meta).plan()
