"""Multi-kernel packages and broadcast elementwise kernels on the GPU.

* broadcast loads (``emmy_pointwise_indexed``): every broadcast form against
  the IR interpreter, bit-exact (f32, f16, f64), and the same plan cut into
  shards with their own element numbering (``first``) gives the same bits;
* the matmul + bias + ReLU package: the fused launch (one matmul with the
  epilogue) gives exactly the bits of the two launches, and both match the
  chain oracle (matmul tolerance: f32 1e-4 relative to max|ref|, f16 output
  one f16 ulp, 2e-3);
* a package written to disk runs through ``Chain.load`` + ``ChainExecutor``;
* at the K3a size (4096 x 8192 x 2048, f16) fused and unfused agree bit for bit.
"""

from __future__ import annotations

import numpy as np
import pytest

from emmy_ir import synth
from emmy_ir.serialize import write_chain
from gpu_util import assert_close
from oracle.interp import make_inputs, run_chain, run_ir
from ptxc import Lowerer
from ptxc.dist import shard_plan

pytestmark = pytest.mark.gpu

BCAST = {
    "row_bias_relu": dict(n=64 * 1024, expr=("relu", ("add", "x0", ("bcast", "bias", 1024, 1, 1024))),
                          shape=[64, 1024]),
    "col_scale": dict(n=300 * 512, expr=("multiply", "x0", ("bcast", "rs", 300, 512, 0)),
                      shape=[300, 512]),
    "middle": dict(n=6 * 40 * 96, expr=("add", "x0", ("bcast", "c", 40, 96, 40)), shape=[6, 40, 96]),
    "tile2_bias": dict(n=96 * 1000, expr=("add", ("multiply", "x0", ("axis", "g", (1,))),
                                          ("axis", "b", (1,))),
                       shape=[96, 1000], tile_shape=[96, 1000]),
    "tile3_mid_gelu": dict(n=5 * 7 * 129, expr=("gelu", ("add", "x0", ("axis", "c", (1,)))),
                           shape=[5, 7, 129], tile_shape=[5, 7, 129]),
    "odd_divisor": dict(n=3 * 1237 * 11, expr=("subtract", "x0", ("bcast", "m", 1237, 11, 1237)),
                        shape=[3 * 1237 * 11]),
}


def _run_plan(plan, host, shards=1):
    import torch
    from ptxc.launch import Executor
    out_name = plan["args"]["out"]
    full = torch.empty(plan["pointwise"]["n"], dtype={"f32": torch.float32, "f16": torch.float16,
                                                      "f64": torch.float64}[plan["pointwise"]["out_dtype"]])
    for r in range(shards):
        sub, sl = shard_plan(plan, r, shards) if shards > 1 else (plan, None)
        ex = Executor(sub)
        if sl:
            ex.upload({n: host[n][o:o + c] for n, (o, c) in sl.items() if n != out_name})
        else:
            ex.upload({n: v for n, v in host.items() if n != out_name})
        ex.launch()
        torch.cuda.synchronize()
        o, c = sl[out_name] if sl else (0, full.numel())
        full[o:o + c] = ex.tensors[out_name].cpu()
    return full.numpy()


@pytest.mark.parametrize("dtype", ["f32", "f16", "f64"])
@pytest.mark.parametrize("case", sorted(BCAST))
def test_broadcast_pointwise_matches_interpreter(case, dtype):
    kop, meta = synth.pointwise(dtype=dtype, **BCAST[case])
    plan = Lowerer(kop, meta).plan()
    assert "input_index" in plan["pointwise"]
    host = make_inputs(meta)
    want = run_ir(kop, meta, host)[plan["args"]["out"]]
    got = _run_plan(plan, host)
    if case == "tile3_mid_gelu":
        tol = {"f32": (1e-5, 1e-6), "f16": (2e-3, 2e-3), "f64": (1e-12, 1e-13)}[dtype]
        assert_close(got, want, *tol, what=case)
    else:
        np.testing.assert_array_equal(got, want, err_msg=case)
    # cut into three shards, each numbering its elements from its own first
    np.testing.assert_array_equal(_run_plan(plan, host, shards=3), got, err_msg=case + " shards")


CHAINS = {
    "f32": dict(M=512, N=384, K=256, kw=dict(dtype="f32")),
    "f32_flat": dict(M=512, N=384, K=256, kw=dict(dtype="f32", axis_form=False)),
    "f16_all": dict(M=512, N=384, K=512, kw=dict(dtype="f16", c_dtype="f16", out_dtype="f16",
                                                 tm=128, tn=128, rm=8, rn=8)),
    "f16_f32mm_f16out": dict(M=256, N=512, K=256, kw=dict(dtype="f16", c_dtype="f32",
                                                          out_dtype="f16", tm=128, tn=128, rm=8, rn=8)),
    "f16_compute_f16": dict(M=512, N=256, K=256, kw=dict(dtype="f16", c_dtype="f16", out_dtype="f16",
                                                         compute="f16", tm=128, tn=128, rm=8, rn=8)),
    "f16_unfusable": dict(M=256, N=256, K=256, kw=dict(dtype="f16", c_dtype="f16", out_dtype="f32",
                                                       compute="f16", tm=128, tn=128, rm=8, rn=8)),
    "f16_small_m": dict(M=128, N=256, K=128, kw=dict(dtype="f16", c_dtype="f16", out_dtype="f16",
                                                     tm=128, tn=128, rm=8, rn=8)),
}


def _host(pairs, scale=None):
    host = {}
    for _, m in pairs:
        for k, v in make_inputs(m).items():
            a = next(x for x in m["args"] if x["name"] == k)
            if not a.get("output") and not a.get("intermediate"):
                host[k] = v
    if scale:
        for k, s in scale.items():
            host[k] = (host[k].astype(np.float64) * s).astype(host[k].dtype)
    return host


def _run_chain(chain, host, fuse):
    import torch
    from ptxc.package import ChainExecutor
    ex = ChainExecutor(chain, fuse=fuse)
    ex.upload(host)
    n = ex.launch()
    torch.cuda.synchronize()
    return ex, n, {k: v.numpy() for k, v in ex.download().items()}


@pytest.mark.parametrize("case", sorted(CHAINS))
def test_fused_chain_matches_two_launches_and_oracle(case):
    from ptxc.package import Chain
    c = CHAINS[case]
    pairs = synth.mm_bias_relu_chain(c["M"], c["N"], c["K"], **c["kw"])
    chain = Chain.from_kernels(pairs)
    # keep |A @ B| near 1 so an f16 product does not overflow
    host = _host(pairs, scale={"A": c["K"] ** -0.5})
    exf, nf, fused = _run_chain(chain, host, True)
    exu, nu, plain = _run_chain(chain, host, False)
    assert nu == 2
    if case == "f16_unfusable":
        assert exf.fused == [] and nf == 2
    else:
        assert exf.fused == [["k_relu__partial", "k_relu"]] and nf == 1
    np.testing.assert_array_equal(fused["out"], plain["out"], err_msg=case)
    ref = run_chain(pairs, host)["out"].astype(np.float64)
    scale = float(np.abs(ref).max())
    if c["kw"]["dtype"] == "f32":
        assert_close(fused["out"], ref, 1e-4, 1e-4 * scale, case)
    else:
        assert_close(fused["out"], ref, 2e-3, 2e-3 * scale, case)


def test_package_from_disk_runs(tmp_path):
    from ptxc.package import Chain
    pairs = synth.mm_bias_relu_chain(256, 256, 128, dtype="f16", c_dtype="f16", out_dtype="f16",
                                     tm=128, tn=128, rm=8, rn=8)
    write_chain(tmp_path, pairs)
    chain = Chain.load(tmp_path)
    host = _host(pairs, scale={"A": 128 ** -0.5})
    ex, n, out = _run_chain(chain, host, True)
    assert n == 1 and list(out) == ["out"]
    ref = run_chain(pairs, host)["out"].astype(np.float64)
    assert_close(out["out"], ref, 2e-3, 2e-3 * float(np.abs(ref).max()), "package")


def test_k3a_size_fused_equals_two_launches():
    from ptxc.package import Chain
    pairs = synth.mm_bias_relu_chain(4096, 8192, 2048, dtype="f16", c_dtype="f16", out_dtype="f16",
                                     tm=128, tn=128, rm=8, rn=8)
    chain = Chain.from_kernels(pairs)
    host = _host(pairs, scale={"A": 2048 ** -0.5})
    _, nf, fused = _run_chain(chain, host, True)
    _, nu, plain = _run_chain(chain, host, False)
    assert (nf, nu) == (1, 2)
    np.testing.assert_array_equal(fused["out"], plain["out"])
    assert np.isfinite(fused["out"].astype(np.float32)).all()
