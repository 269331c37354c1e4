"""The reference compiler's own PTX on the B200, beside the B200 kernels.

``oracle/make_ref_ptx.py`` (run where the reference checkout exists) emits,
with the unmodified reference compiler, the PTX of all 46 reference fixtures
and of the benchmark configurations into ``oracle/_ref/``; ``oracle/ref_ptx.py``
launches it as the reference harness does.  Checked here:

* the reference PTX reproduces the reference's goldens on this GPU (fixture
  rtol/atol) -- so the comparison below is against the real reference;
* on every fixture, the B200 kernels match the reference PTX's output within
  the fixture's rtol/atol (``|ours - ref| <= atol + rtol * |ref|``);
* on the full-size benchmark configurations, the B200 kernels are within the
  north-star bound of float64 (``tests/parity.py``: f32 1e-5, f16 with f32
  accumulation 1e-3, f64 1e-12, each relative to the family's error scale),
  and within twice that bound of the reference PTX's own output.

Skipped when ``oracle/_ref`` has not been generated.
"""

from __future__ import annotations

import numpy as np
import pytest

from emmy_ir import synth
from golden import replicas
from gpu_util import run_on_gpu, shaped
from oracle import formulas as F
from oracle import ref_ptx
from oracle.interp import make_inputs
from parity import check

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not ref_ptx.names(), reason="oracle/_ref not generated")]

FIXTURES = [f for f in replicas.replica_ids() if ref_ptx.available(f)]


def _bound_check(ours, ref, rtol, atol, what):
    ours = np.asarray(ours, dtype=np.float64).reshape(-1)
    ref = np.asarray(ref, dtype=np.float64).reshape(-1)
    assert ours.shape == ref.shape, what
    err = np.abs(ours - ref)
    bound = atol + rtol * np.abs(ref)
    bad = err > bound
    assert not bad.any(), (f"{what}: {int(bad.sum())} of {err.size} outside atol {atol:.3g} + "
                           f"rtol {rtol} * |ref|; worst |d| {float(err.max()):.3g}")


@pytest.mark.parametrize("fid", FIXTURES)
def test_reference_ptx_reproduces_its_golden(fid):
    k = ref_ptx.RefKernel(fid)
    try:
        host = make_inputs({"args": replicas.table()[fid]["args"]})
        out = k.run(host)
    finally:
        k.close()
    worst, msg = replicas.compare(fid, out[replicas.table()[fid]["output"]])
    assert worst <= 0, "reference PTX: " + msg


@pytest.mark.parametrize("fid", FIXTURES)
def test_b200_kernel_matches_reference_ptx(fid):
    entry = replicas.table()[fid]
    k = ref_ptx.RefKernel(fid)
    try:
        ref = k.run(make_inputs({"args": entry["args"]}))[entry["output"]]
    finally:
        k.close()
    kop, meta, names = replicas.build(fid)
    out_name = next(a["name"] for a in meta["args"] if a.get("output"))
    _, _, out = run_on_gpu(kop, meta, replicas.fixture_inputs(fid, meta, names))
    _bound_check(out[out_name], ref, entry["rtol"], entry["atol"], fid)


# benchmark configurations (builders shared with make_ref_ptx): per case the
# float64 reference, the error scale and the arithmetic of ``tests/parity.py``
def _bench_ref(name, x):
    """(float64 reference, scale or None for |ref|, arithmetic dtype, output dtype)."""
    f64 = lambda a: np.asarray(a, dtype=np.float64)  # noqa: E731
    if name == "K1_rmsnorm":
        return F.rmsnorm(x["x"], x["w"], 1e-6, out_dtype=np.float64), None, "f32", "f32"
    if name == "K2a_softmax":
        return F.softmax(x["x"], out_dtype=np.float64), None, "f32", "f32"
    if name == "K2b_layernorm":
        return (F.layernorm(x["x"], x["gamma"], x["beta"], 1e-5, out_dtype=np.float64),
                F.layernorm_abs_scale(x["x"], x["gamma"], x["beta"], 1e-5), "f32", "f32")
    if name == "K4b_matvec_f64":
        return F.matvec(x["A"], x["v"]), np.abs(f64(x["A"])) @ np.abs(f64(x["v"])), "f64", "f64"
    if name == "K4a_splitk_f32":
        return (F.matmul(x["A"], x["B"], out_dtype=np.float64), F.matmul_abs_bound(x["A"], x["B"]),
                "f32", "f32")
    if name == "K3a_gemm_f16":
        return (F.matmul(x["A"], x["B"], x["bias"], True, out_dtype=np.float64),
                F.matmul_abs_bound(x["A"], x["B"], x["bias"]), "f16", "f16")
    if name == "K3b_bmm_f16":
        return (np.matmul(f64(x["A"]), f64(x["B"])),
                np.matmul(np.abs(f64(x["A"])), np.abs(f64(x["B"]))), "f16", "f16")
    if name == "K5_attention_f16":
        sc = 1.0 / 11.313708498984761
        return (F.attention_bhsd(x["q"], x["k"], x["v"], sc, out_dtype=np.float64),
                F.attention_abs_scale(x["q"], x["k"], x["v"], sc), "f16", "f16")
    if name == "F8a_pointwise_add":
        # correctly rounded f32 add: bit-exact
        return ((x["x0"].astype(np.float32) + x["x1"].astype(np.float32)).astype(np.float64),
                None, "f32", "f32")
    raise KeyError(name)


BENCH_NAMES = ["K1_rmsnorm", "K2a_softmax", "K2b_layernorm", "K4b_matvec_f64", "K4a_splitk_f32",
               "K3a_gemm_f16", "K3b_bmm_f16", "K5_attention_f16", "F8a_pointwise_add"]


@pytest.mark.parametrize("name", [n for n in BENCH_NAMES if ref_ptx.available(n)])
def test_b200_kernel_matches_reference_ptx_at_benchmark_size(name):
    """At the full benchmark size: the B200 kernel is within the north-star
    bound of float64; the reference's own PTX output is logged against the same
    bound; the two differ by at most the sum of their bounds (bit-exact for the
    correctly rounded add)."""
    from oracle import make_ref_ptx
    kop, meta = make_ref_ptx.BENCH_CASES[name](synth)
    host = synth.make_inputs(meta)
    k = ref_ptx.RefKernel(name)
    try:
        out_name = next(a["name"] for a in meta["args"] if a.get("output"))
        ref = k.run(host)[out_name]
    finally:
        k.close()
    _, _, out = run_on_gpu(kop, meta, host)
    x = shaped(meta, host)
    want, scale, dt, odt = _bench_ref(name, x)
    ours = np.asarray(out[out_name], dtype=np.float64).reshape(want.shape)
    theirs = np.asarray(ref, dtype=np.float64).reshape(want.shape)
    if name == "F8a_pointwise_add":
        check(ours, want, None, case=f"bench {name}", family="pointwise", dtype="f32", rtol=0.0,
              floor=0.0)
        assert np.array_equal(ours, theirs), name
        return
    check(ours, want, scale, case=f"bench {name}", family=name, dtype=dt, out_dtype=odt)
    try:
        check(theirs, want, scale, case=f"bench {name} (reference PTX)", family=name, dtype=dt,
              out_dtype=odt)
    except AssertionError:
        pass            # logged only: the bar here is the B200 kernel, not the reference
    sc = np.abs(want) if scale is None else scale
    check(ours, theirs, 2 * sc, case=f"bench {name} vs reference PTX", family=name, dtype=dt,
          out_dtype=odt, u_mult=2.0)
