"""The reference compiler's own PTX on the B200, beside the B200 kernels.

``oracle/make_ref_ptx.py`` (run where the reference checkout exists) emits,
with the unmodified reference compiler, the PTX of all 46 reference fixtures
and of the benchmark configurations into ``oracle/_ref/``; ``oracle/ref_ptx.py``
launches it as the reference harness does.  Checked here:

* the reference PTX reproduces the reference's goldens on this GPU (fixture
  rtol/atol) -- so the comparison below is against the real reference;
* on every fixture, the B200 kernels match the reference PTX's output within
  the fixture's rtol/atol (``|ours - ref| <= atol + rtol * |ref|``);
* on the full-size benchmark configurations, the B200 kernels match the
  reference PTX within the family tolerance written beside each case.

Skipped when ``oracle/_ref`` has not been generated.
"""

from __future__ import annotations

import numpy as np
import pytest

from emmy_ir import synth
from golden import replicas
from gpu_util import run_on_gpu
from oracle import ref_ptx
from oracle.interp import make_inputs

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


# benchmark configurations: builder (shared with make_ref_ptx) and tolerance (rtol, atol as a
# fraction of max|ref|), per family
BENCH_TOL = {
    "K1_rmsnorm": (1e-5, 1e-6),          # f32 row norm: rsqrt/recip rounding
    "K2a_softmax": (1e-5, 1e-6),         # f32: ex2.approx vs __expf, one-pass vs online
    "K2b_layernorm": (1e-5, 1e-6),       # f32: two-pass vs two-moment variance
    "K4b_matvec_f64": (1e-12, 1e-13),    # f64 reduction order
    "K4a_splitk_f32": (1e-4, 1e-5),      # f32 split-K: summation order of 65536 products
    "K3a_gemm_f16": (2e-3, 2e-3),        # f16 output: one f16 ulp
    "K3b_bmm_f16": (2e-3, 2e-3),
    "K5_attention_f16": (4e-3, 2e-3),    # f16 P on the tensor cores vs f32 P V in the reference
    "F8a_pointwise_add": (0.0, 0.0),     # correctly rounded add
}


@pytest.mark.parametrize("name", [n for n in BENCH_TOL if ref_ptx.available(n)])
def test_b200_kernel_matches_reference_ptx_at_benchmark_size(name):
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
    rtol, atol_frac = BENCH_TOL[name]
    _bound_check(out[out_name], ref, rtol, atol_frac * float(np.abs(ref).max()), name)
