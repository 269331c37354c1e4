"""Multi-kernel packages, broadcast elementwise inputs and matmul epilogue
fusion -- host side (no GPU).

* ``resolve_ir`` follows the reference resolver and its unit tests
  (``tools/irfiles.py:17-29``; ``tests/test_lowering.py:459-475``): the exact
  entry file beats a shared prefix, a lone file is taken, a missing entry
  among several is an error.
* a package written to disk loads back, compiles kernel by kernel, and names
  its host inputs and final outputs as the harness does
  (``tools/localrun.py:160-195``);
* the fusion rules: which chains run as one matmul with an epilogue and which
  stay two launches (or get a dtype conversion in between);
* broadcast loads (``bias[e % N]``, ``scale[e // N]``, a middle axis, a
  multi-axis Tile) become plans with ``input_index``; pipeline chunks and
  shards of such plans keep the element numbering (``first``);
* the chain oracle reproduces a float64 formula.
"""

from __future__ import annotations

import numpy as np
import pytest

from emmy_ir import synth
from emmy_ir.serialize import write_chain
from oracle.interp import make_inputs, run_chain
from ptxc import CompileError, Lowerer
from ptxc.dist import shard_plan
from ptxc.package import Chain, IRError, resolve_ir, schedule


def test_resolve_exact_entry_beats_prefix(tmp_path):
    (tmp_path / "k_sum_1.ir.json").write_text("{}")
    (tmp_path / "k_sum_1__partial.ir.json").write_text("{}")
    assert resolve_ir(tmp_path, "k_sum_1").name == "k_sum_1.ir.json"
    assert resolve_ir(tmp_path, "k_sum_1__partial").name == "k_sum_1__partial.ir.json"


def test_resolve_single_file_and_missing_entry(tmp_path):
    (tmp_path / "a.ir.json").write_text("{}")
    assert resolve_ir(tmp_path, "anything").name == "a.ir.json"
    (tmp_path / "b.ir.json").write_text("{}")
    with pytest.raises(IRError, match="no IR for entry 'c'"):
        resolve_ir(tmp_path, "c")
    (tmp_path / "empty").mkdir()
    with pytest.raises(IRError, match="no .ir.json"):
        resolve_ir(tmp_path / "empty", "c")


def _chain(**kw):
    if kw.get("dtype", "f32") == "f16":
        kw = dict(tm=128, tn=128, rm=8, rn=8, **kw)
    return synth.mm_bias_relu_chain(256, 128, 64, **kw)


def test_package_round_trip(tmp_path):
    pairs = _chain()
    write_chain(tmp_path, pairs)
    ch = Chain.load(tmp_path)
    assert [s["entry"] for s in ch.steps] == ["k_relu__partial", "k_relu"]
    assert [s["final"] for s in ch.steps] == [False, True]
    assert [s["plan"]["family"] for s in ch.steps] == ["gemm_f32", "pointwise"]
    assert sorted(ch.host_inputs()) == ["A", "B", "bias"]
    assert ch.outputs() == ["out"]


def test_package_with_a_foreign_kernel_name_is_refused(tmp_path):
    pairs = _chain()
    write_chain(tmp_path, pairs)
    (tmp_path / "k_relu.ir.json").rename(tmp_path / "k_other.ir.json")
    with pytest.raises((IRError, CompileError)):
        Chain.load(tmp_path)


def _families(launches):
    return [(p["family"], p.get("gemm", {}).get("epilogue"), p.get("gemm", {}).get("out_dtype"))
            for p, _ in launches]


@pytest.mark.parametrize("kw, fused", [
    (dict(dtype="f32"), [("gemm_f32", 3, None)]),
    (dict(dtype="f32", axis_form=False), [("gemm_f32", 3, None)]),
    (dict(dtype="f32", relu=False), [("gemm_f32", 1, None)]),
    (dict(dtype="f32", bias=False), [("gemm_f32", 2, None)]),
    (dict(dtype="f16", c_dtype="f16", out_dtype="f16"), [("gemm_f16", 7, 1)]),
    (dict(dtype="f16", c_dtype="f32", out_dtype="f16"), [("gemm_f16", 3, 1)]),
    (dict(dtype="f16", c_dtype="f32", out_dtype="f32"), [("gemm_f16", 3, 0)]),
    (dict(dtype="f16", c_dtype="f16", out_dtype="f16", compute="f16"), [("gemm_f16", 7, 1)]),
    (dict(dtype="f16", c_dtype="f16", out_dtype="f32", relu=False), [("gemm_f16", 5, 0)]),
])
def test_fusable_chains_become_one_matmul(kw, fused):
    ch = Chain.from_kernels(_chain(**kw))
    launches = schedule(ch, fuse=True)
    assert _families(launches) == fused
    plan = launches[0][0]
    assert plan["args"]["c"] == "out" and plan["fused_from"] == ["k_relu__partial", "k_relu"]
    assert "mm" not in plan["tensors"]
    assert [p["family"] for p, _ in schedule(ch, fuse=False)] == [ch.steps[0]["plan"]["family"],
                                                                  "pointwise"]


def test_chains_that_stay_two_launches():
    # the sum is rounded to f16 inside the elementwise kernel but stored as f32
    ch = Chain.from_kernels(_chain(dtype="f16", c_dtype="f16", out_dtype="f32", compute="f16"))
    assert [p["family"] for p, _ in schedule(ch)] == ["gemm_f16", "pointwise"]
    # an f32 matmul cannot write f16
    ch = Chain.from_kernels(_chain(dtype="f32", out_dtype="f16"))
    assert [p["family"] for p, _ in schedule(ch)] == ["gemm_f32", "pointwise"]
    # the product is itself a final output
    pairs = _chain()
    pairs[0][1]["final"] = True
    assert [p["family"] for p, _ in schedule(Chain.from_kernels(pairs))] == ["gemm_f32", "pointwise"]
    # split-K atomics
    pairs = synth.mm_bias_relu_chain(128, 128, 256, splits=4)
    assert [p["family"] for p, _ in schedule(Chain.from_kernels(pairs))] == ["gemm_f32", "pointwise"]


def test_retyped_intermediate_gets_a_conversion_launch():
    pairs = _chain(dtype="f32")
    for a in pairs[1][1]["args"]:
        if a["name"] == "mm":
            a["dtype"] = "f16"
    # kernel 2 re-declares mm as f16: its IR loads it as f16 too
    kop, meta = synth.pointwise(256 * 128, ("relu", ("add", "mm", ("axis", "bias", (1,)))), "f32",
                                shape=[256, 128], entry="k_relu", tile_shape=[256, 128],
                                dtypes={"mm": "f16", "bias": "f32"})
    for a in meta["args"]:
        if a["name"] == "mm":
            a["intermediate"] = True
    pairs[1] = (kop, meta)
    launches = schedule(Chain.from_kernels(pairs))
    fams = [p["family"] for p, _ in launches]
    assert fams == ["gemm_f32", "pointwise", "pointwise"]
    conv, bind = launches[1]
    assert conv["pointwise"]["out_dtype"] == "f16" and "mm@f16" in bind.values()
    assert launches[2][1]["mm"] == "mm@f16"


BCAST = {
    "row_bias": (synth.pointwise, dict(n=64 * 128, expr=("relu", ("add", "x0", ("bcast", "bias", 128, 1, 128))),
                                      shape=[64, 128]), [[0, 0], [1, 128]]),
    "col_scale": (synth.pointwise, dict(n=64 * 128, expr=("multiply", "x0", ("bcast", "rs", 64, 128, 0)),
                                       shape=[64, 128]), [[0, 0], [128, 0]]),
    "middle": (synth.pointwise, dict(n=4 * 8 * 16, expr=("add", "x0", ("bcast", "c", 8, 16, 8)),
                                    shape=[4, 8, 16]), [[0, 0], [16, 8]]),
    "tile2_bias": (synth.pointwise, dict(n=64 * 128, expr=("add", "x0", ("axis", "bias", (1,))),
                                        shape=[64, 128], tile_shape=[64, 128]), [[0, 0], [1, 128]]),
    "tile2_rows": (synth.pointwise, dict(n=64 * 128, expr=("multiply", "x0", ("axis", "rs", (0,))),
                                        shape=[64, 128], tile_shape=[64, 128]), [[0, 0], [128, 0]]),
    "tile3_mid": (synth.pointwise, dict(n=4 * 8 * 16, expr=("add", "x0", ("axis", "c", (1,))),
                                       shape=[4, 8, 16], tile_shape=[4, 8, 16]), [[0, 0], [16, 8]]),
}


@pytest.mark.parametrize("case", sorted(BCAST))
def test_broadcast_loads_plan(case):
    fn, kw, index = BCAST[case]
    kop, meta = fn(**kw)
    g = Lowerer(kop, meta).plan()["pointwise"]
    assert g["input_index"] == index and g["first"] == 0


def test_multi_axis_tile_without_broadcast_is_plain():
    kop, meta = synth.pointwise(64 * 128, ("add", "x0", "x1"), shape=[64, 128], tile_shape=[64, 128])
    g = Lowerer(kop, meta).plan()["pointwise"]
    assert "input_index" not in g and g["inputs"] == ["x0", "x1"]


def test_two_axis_broadcast_of_a_three_axis_tile_is_refused():
    kop, meta = synth.pointwise(4 * 8 * 16, ("add", "x0", ("axis", "c", (0, 2))), shape=[4, 8, 16],
                                tile_shape=[4, 8, 16])
    with pytest.raises(CompileError, match="broadcast"):
        Lowerer(kop, meta).plan()


def test_broadcast_past_the_tensor_is_refused():
    # bias of 100 elements read at e % 128
    kop, meta = synth.pointwise(64 * 128, ("add", "x0", ("bcast", "bias", 128, 1, 128)), shape=[64, 128])
    for a in meta["args"]:
        if a["name"] == "bias":
            a["shape"] = [100]
    with pytest.raises(CompileError, match="past"):
        Lowerer(kop, meta).plan()


def test_shards_of_a_broadcast_plan_keep_element_numbers():
    kop, meta = synth.pointwise(64 * 128, ("add", "x0", ("bcast", "bias", 128, 1, 128)), shape=[64, 128])
    plan = Lowerer(kop, meta).plan()
    firsts = []
    for r in range(3):
        sub, sl = shard_plan(plan, r, 3)
        assert sl["bias"] == (0, 128)
        assert sl["x0"][0] == sub["pointwise"]["first"]
        firsts.append((sub["pointwise"]["first"], sub["pointwise"]["n"]))
    assert firsts[0][0] == 0 and sum(n for _, n in firsts) == 64 * 128
    # a tensor read both whole and broadcast cannot be cut into element ranges
    kop, meta = synth.pointwise(128, ("add", "x0", ("bcast", "x0", 128, 2, 0)), shape=[128])
    with pytest.raises(ValueError, match="both"):
        shard_plan(Lowerer(kop, meta).plan(), 0, 2)


def test_chain_oracle_matches_float64_formula():
    pairs = synth.mm_bias_relu_chain(64, 128, 32)
    host = {}
    for _, m in pairs:
        for k, v in make_inputs(m).items():
            a = next(x for x in m["args"] if x["name"] == k)
            if not a.get("output") and not a.get("intermediate"):
                host[k] = v
    out = run_chain(pairs, host)
    A = host["A"].reshape(64, 32).astype(np.float64)
    B = host["B"].reshape(32, 128).astype(np.float64)
    ref = np.maximum(A @ B + host["bias"].astype(np.float64), 0)
    np.testing.assert_allclose(out["out"].reshape(64, 128), ref, rtol=1e-5, atol=1e-5)
    assert set(out) == {"mm", "out"}
