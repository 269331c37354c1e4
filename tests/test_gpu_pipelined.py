"""``Executor.run_pipelined``: host in, host out, copies overlapping kernels.

The plan runs in chunks along its shard axis with H2D, kernels and D2H on
three streams.  Checked against the plain ``upload -> launch -> download``
path of the same plan: bit-exact where a chunk runs the same kernel on the
same rows (row norms, softmax, pointwise, attention heads); within the matmul
tolerance where a smaller M changes the tile or split-K choice.  Chunk counts
include one that does not divide the shard axis, and a split-K matmul whose
atomic partial sums add onto a C the host provides (C is then uploaded too).
"""

from __future__ import annotations

import numpy as np
import pytest

from emmy_ir import synth
from gpu_util import assert_close, plan_of

pytestmark = pytest.mark.gpu


def _pinned(host):
    import torch
    return {k: torch.from_numpy(np.ascontiguousarray(v)).pin_memory() for k, v in host.items()}


def _both(kop, meta, chunks, host=None):
    import torch
    from ptxc.launch import Executor
    plan = plan_of(kop, meta)
    host = host if host is not None else synth.make_inputs(meta)
    ex = Executor(plan)
    ex.upload(host)
    ex.launch()
    torch.cuda.synchronize()
    want = {k: v.numpy().copy() for k, v in ex.download().items()}
    pin = _pinned(host)
    ex2 = Executor(plan)
    for n in plan["outputs"]:                     # stale device contents must not leak through
        ex2.tensors[n].fill_(float("nan"))
    out = {n: torch.empty(ex2.tensors[n].numel(), dtype=ex2.tensors[n].dtype).pin_memory()
           for n in plan["outputs"]}
    ex2.run_pipelined(pin, out, chunks=chunks)
    torch.cuda.synchronize()
    return plan, want, {k: v.numpy() for k, v in out.items()}


EXACT = {
    "softmax": lambda: synth.softmax([8, 4, 64, 512]),
    "layernorm": lambda: synth.layernorm(1000, 1024),
    "rmsnorm": lambda: synth.rmsnorm(777, 512, eps=1e-6),
    "reduce_mean": lambda: synth.reduce([300, 2048], op="mean"),
    "matvec_f64": lambda: synth.matvec(513, 4096),
    "pointwise_gelu_f16": lambda: synth.pointwise(
        1 << 20, ("gelu_tanh", "x0"), "f16"),
    "attention_f16": lambda: synth.attention(2, 8, 256, 128, dtype="f16"),
    "softmax_f16_rows": lambda: synth.retype(*synth.softmax([300, 1024]), "f16", acc="f32"),
    "broadcast_bias": lambda: synth.pointwise(512 * 768, ("add", "x0", ("bcast", "b", 768, 1, 768)),
                                              "f32", shape=[512, 768]),
}


@pytest.mark.parametrize("chunks", [1, 3, 8])
@pytest.mark.parametrize("case", sorted(EXACT))
def test_pipelined_matches_plain_exactly(case, chunks):
    kop, meta = EXACT[case]()
    plan, want, got = _both(kop, meta, chunks)
    for n in plan["outputs"]:
        np.testing.assert_array_equal(got[n], want[n], err_msg=f"{case} chunks={chunks}")


@pytest.mark.parametrize("chunks", [2, 5])
def test_pipelined_gemm_f16_rows_and_batches(chunks):
    kop, meta = synth.matmul(1024, 512, 512, dtype="f16", out_dtype="f16", bias=True, relu=True,
                             tm=128, tn=128, rm=8, rn=8)
    plan, want, got = _both(kop, meta, chunks)
    assert_close(got["C"], want["C"], 2e-3, 2e-3, "gemm f16 row chunks")
    kop, meta = synth.matmul(256, 256, 256, batch=6, dtype="f16", out_dtype="f16",
                             tm=128, tn=128, rm=8, rn=8)
    plan, want, got = _both(kop, meta, chunks)
    assert_close(got["C"], want["C"], 2e-3, 2e-3, "bmm f16 batch chunks")


def test_pipelined_splitk_accumulates_onto_host_c():
    kop, meta = synth.matmul(256, 128, 4096, splits=8, tm=64, tn=64, rm=4, rn=4)
    meta = dict(meta, zero_outputs=[])             # partial sums add onto the C given
    host = synth.make_inputs(meta)
    host["C"] = np.random.default_rng(5).standard_normal(host["C"].size).astype(np.float32)
    plan, want, got = _both(kop, meta, 4, host=host)
    assert plan["gemm"]["accumulate"]
    ref = host["C"].astype(np.float64) + (host["A"].reshape(256, 4096).astype(np.float64)
                                          @ host["B"].reshape(4096, 128)).reshape(-1)
    assert_close(want["C"], ref, 1e-4, 1e-4 * np.abs(ref).max(), "plain split-K")
    assert_close(got["C"], ref, 1e-4, 1e-4 * np.abs(ref).max(), "pipelined split-K")


def test_pipelined_calls_chain_without_join():
    """Two plans queued with ``join=False`` then ``join=True``, run twice in a row."""
    import torch
    from ptxc.launch import Executor
    cases = [synth.softmax([64, 4096]), synth.layernorm(512, 1024)]
    plans = [plan_of(k, m) for k, m in cases]
    hosts = [synth.make_inputs(m) for _, m in cases]
    execs = [Executor(p) for p in plans]
    outs = [{n: torch.empty(ex.tensors[n].numel(), dtype=ex.tensors[n].dtype).pin_memory()
             for n in p["outputs"]} for ex, p in zip(execs, plans)]
    pins = [_pinned(h) for h in hosts]
    for _ in range(2):
        for j, (ex, h, o) in enumerate(zip(execs, pins, outs)):
            ex.run_pipelined(h, o, chunks=4, join=(j == 1))
    torch.cuda.synchronize()
    for (kop, meta), h, o in zip(cases, hosts, outs):
        plan, want, _ = _both(kop, meta, 1, host=h)
        for n in plan["outputs"]:
            np.testing.assert_array_equal(o[n].numpy(), want[n])
