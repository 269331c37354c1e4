"""GPU parity of the memory-bound families (reduce / rownorm / softmax / matvec).

Each case is IR (the reference fixture shapes, the benchmark configurations
and edge cases), compiled to a plan by the matcher and run through the C-ABI.
Results are compared with the float64 oracle (``oracle.formulas``) and, for
small cases, with the statement-level IR interpreter (``oracle.interp``).

Tolerances (per output element, ``tests/parity.py``; the north star's 1e-5
for f32 and 1e-12 for f64):
* softmax, rms and l2 norm (products and sums of positive terms): plain
  relative, ``|got - ref| <= 1e-5 * |ref|`` (+1e-30 for flushed denormals);
* layer norm: ``|got - ref| <= 1e-5 * ((|x| + |mean|) * rstd * |gamma| +
  |beta|)``, the magnitude of the terms the output is formed from;
* f32 reductions: ``|got - ref| <= 1e-5 * sum|x|`` over the reduced slice
  (the scale of the sum), exact for max;
* f64 matvec: ``|got - ref| <= 1e-12 * (|A| @ |v|)``.
"""

from __future__ import annotations

import numpy as np
import pytest

from emmy_ir import synth
from gpu_util import run_on_gpu, shaped
from oracle import formulas as F
from oracle.interp import run_ir
from parity import check

pytestmark = pytest.mark.gpu

RTOL = 1e-5


def _elementwise(got, ref, what, family, scale=None):
    check(got.reshape(ref.shape), ref, scale, case=what, family=family, dtype="f32")


ROWNORM_CASES = [
    ("rms_fixture_128x512", lambda: synth.rmsnorm(128, 512, eps=1e-5), "rms"),
    ("rms_fixture_16x2048", lambda: synth.rmsnorm(16, 2048, eps=1e-5), "rms"),
    ("rms_K1_4096x512", lambda: synth.rmsnorm(4096, 512, eps=1e-6,
                                              w_init={"dist": "uniform", "low": 0.5, "high": 1.5}), "rms"),
    ("rms_noweight_odd_37x300", lambda: synth.rmsnorm(37, 300, weight=False), "rms"),
    ("rms_long_3x40000", lambda: synth.rmsnorm(3, 40000), "rms"),
    ("rms_one_col", lambda: synth.rmsnorm(64, 1), "rms"),
    ("l2_fixture_128x256", lambda: synth.l2norm(128, 256), "l2"),
    ("l2_odd_5x777", lambda: synth.l2norm(5, 777), "l2"),
    ("ln_K2b_16384x1024", lambda: synth.layernorm(16384, 1024, eps=1e-5,
                                                  g_init={"dist": "uniform", "low": 0.5, "high": 1.5},
                                                  b_init={"dist": "normal", "std": 0.1}), "ln"),
    ("ln_noaffine_9x4096", lambda: synth.layernorm(9, 4096, affine=False), "ln"),
    ("ln_odd_7x1001", lambda: synth.layernorm(7, 1001), "ln"),
    ("ln_long_2x50000", lambda: synth.layernorm(2, 50000), "ln"),
]


@pytest.mark.parametrize("name,make,kind", ROWNORM_CASES, ids=[c[0] for c in ROWNORM_CASES])
def test_rownorm(name, make, kind):
    kop, meta = make()
    plan, host, out = run_on_gpu(kop, meta)
    assert plan["family"] == "rownorm"
    x = shaped(meta, host)
    eps = {a["name"]: a["data"][0] for a in meta["args"] if "data" in a}
    scale = None
    if kind == "rms":
        ref = F.rmsnorm(x["x"], x.get("w"), eps["add_c1"], out_dtype=np.float64)
    elif kind == "l2":
        ref = F.l2norm(x["x"], out_dtype=np.float64)
    else:
        ref = F.layernorm(x["x"], x.get("gamma"), x.get("beta"), eps["ln_eps"],
                          out_dtype=np.float64)
        scale = F.layernorm_abs_scale(x["x"], x.get("gamma"), x.get("beta"), eps["ln_eps"])
    _elementwise(out["y"], ref, f"rownorm {name}", {"rms": "rmsnorm", "l2": "l2norm",
                                                     "ln": "layernorm"}[kind], scale)


SOFTMAX_CASES = [
    ("fixture_128x384", lambda: synth.softmax([128, 384]), -1),
    ("fixture_32x1024", lambda: synth.softmax([32, 1024]), -1),
    ("fixture_16x2048", lambda: synth.softmax([16, 2048]), -1),
    ("fixture_dim0_128x64", lambda: synth.softmax([128, 64], dim=0), 0),
    ("K2a_4d_32x16x512x512", lambda: synth.softmax([32, 16, 512, 512],
                                                   x_init={"dist": "normal", "std": 2.0}), -1),
    ("odd_61x333", lambda: synth.softmax([61, 333]), -1),
    ("one_col_64x1", lambda: synth.softmax([64, 1]), -1),
    ("long_3x70000", lambda: synth.softmax([3, 70000]), -1),
    ("dim0_odd_33x17", lambda: synth.softmax([33, 17], dim=0), 0),
]


@pytest.mark.parametrize("name,make,dim", SOFTMAX_CASES, ids=[c[0] for c in SOFTMAX_CASES])
def test_softmax(name, make, dim):
    kop, meta = make()
    plan, host, out = run_on_gpu(kop, meta)
    assert plan["family"] == "softmax"
    x = shaped(meta, host)["x"]
    ref = F.softmax(x, axis=dim, out_dtype=np.float64)
    _elementwise(out["y"], ref, f"softmax {name}", "softmax")
    if np.prod(x.shape) <= 1 << 16:
        # the interpreter is itself an f32 evaluation: the two differ by at
        # most the sum of their errors
        interp = run_ir(kop, meta, host)["y"].reshape(ref.shape)
        check(out["y"].reshape(ref.shape), interp.astype(np.float64), ref,
              case=f"softmax {name} vs interpreter", family="softmax", dtype="f32", rtol=2e-5)


REDUCE_CASES = [
    ("sum_100000", lambda: synth.reduce([100000], None, "sum"), None, "sum"),
    ("sum_4096", lambda: synth.reduce([4096], None, "sum"), None, "sum"),
    ("sum_65536_t256", lambda: synth.reduce([65536], None, "sum", block=256), None, "sum"),
    ("sum_131072_t512", lambda: synth.reduce([131072], None, "sum", block=512), None, "sum"),
    ("sum_3d_last", lambda: synth.reduce([8, 32, 256], -1, "sum"), -1, "sum"),
    ("mean_96x1000", lambda: synth.reduce([96, 1000], -1, "mean"), -1, "mean"),
    ("sum_48x300", lambda: synth.reduce([48, 300], -1, "sum"), -1, "sum"),
    ("sum_17x777", lambda: synth.reduce([17, 777], -1, "sum"), -1, "sum"),
    ("sum_dim0_64x128", lambda: synth.reduce([64, 128], 0, "sum"), 0, "sum"),
    ("sum_mid_8x64x32", lambda: synth.reduce([8, 64, 32], 1, "sum"), 1, "sum"),
    ("max_33x1000", lambda: synth.reduce([33, 1000], -1, "max"), -1, "max"),
    ("max_dim0_19x40", lambda: synth.reduce([19, 40], 0, "max"), 0, "max"),
    ("sum_long_3M", lambda: synth.reduce([3_000_001], None, "sum", block=1024), None, "sum"),
    ("mean_many_rows_20000x64", lambda: synth.reduce([20000, 64], -1, "mean"), -1, "mean"),
]


@pytest.mark.parametrize("name,make,axis,op", REDUCE_CASES, ids=[c[0] for c in REDUCE_CASES])
def test_reduce(name, make, axis, op):
    kop, meta = make()
    plan, host, out = run_on_gpu(kop, meta)
    assert plan["family"] == "reduce"
    x = shaped(meta, host)["x"].astype(np.float64)
    ref = np.asarray(F.reduce(x, axis, op, out_dtype=np.float64)).reshape(-1)
    got = out["y"].astype(np.float64).reshape(-1)
    if op == "max":
        assert np.array_equal(got, ref.astype(np.float32).astype(np.float64)), name
        return
    scale = np.asarray(np.abs(x).sum(axis=axis)).reshape(-1)
    if op == "mean":
        scale = scale / (x.size // max(1, ref.size))
    check(got, ref, scale, case=f"reduce {name}", family="reduce", dtype="f32")


@pytest.mark.parametrize("rows,cols", [(16384, 16384), (1000, 1001), (3, 70)])
def test_matvec_f64(rows, cols):
    kop, meta = synth.matvec(rows, cols)
    plan, host, out = run_on_gpu(kop, meta)
    assert plan["family"] == "matvec"
    x = shaped(meta, host)
    ref = F.matvec(x["A"], x["v"])
    check(out["y"], ref, np.abs(x["A"]) @ np.abs(x["v"]), case=f"matvec_f64 {rows}x{cols}",
          family="matvec", dtype="f64")


def test_unaligned_pointers_take_the_scalar_path():
    """A row view that starts 4 bytes into its buffer must still be exact."""
    import ctypes
    import torch
    from ptxc.launch import load_library
    lib = load_library()
    x = torch.randn(65 * 256 + 1, device="cuda")
    y = torch.zeros_like(x)
    xv, yv = x[1:], y[1:]
    rc = lib.emmy_softmax_f32(ctypes.c_void_p(xv.data_ptr()), ctypes.c_void_p(yv.data_ptr()),
                              65, 256, 1, None)
    assert rc == 0
    torch.cuda.synchronize()
    ref = torch.softmax(xv.double().view(65, 256), dim=-1)
    assert torch.allclose(yv.view(65, 256).double(), ref, rtol=1e-5, atol=1e-9)
    assert y[0].item() == 0.0


def test_device_status_starts_clear():
    import ctypes
    from ptxc.launch import load_library
    code = ctypes.c_int(-1)
    assert load_library().emmy_get_device_status(ctypes.byref(code), None) == 0
    assert code.value == 0
