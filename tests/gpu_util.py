"""Helpers for the GPU parity tests: plan -> C-ABI launch -> numpy outputs."""

from __future__ import annotations

import numpy as np

from emmy_ir import synth
from ptxc import Lowerer


def plan_of(kop, meta):
    return Lowerer(kop, meta).plan()


def run_on_gpu(kop, meta, inputs=None):
    """Compile the IR to a plan, run it through libemmyb200.so, return (plan, inputs, outputs)."""
    import torch
    from ptxc.launch import Executor
    plan = plan_of(kop, meta)
    host = inputs if inputs is not None else synth.make_inputs(meta)
    ex = Executor(plan)
    ex.upload(host)
    ex.launch()
    torch.cuda.synchronize()
    outs = {k: v.numpy() for k, v in ex.download().items()}
    return plan, host, outs


def shaped(meta, arrays):
    shp = {a["name"]: tuple(a["shape"]) for a in meta["args"]}
    return {k: v.reshape(shp[k]) for k, v in arrays.items()}


def assert_close(got, want, rtol, atol, what=""):
    got = np.asarray(got, dtype=np.float64)
    want = np.asarray(want, dtype=np.float64)
    assert got.shape == want.shape, (got.shape, want.shape)
    err = np.abs(got - want)
    bound = rtol * np.abs(want) + atol
    bad = err > bound
    if bad.any():
        i = np.unravel_index(np.argmax(err - bound), err.shape)
        raise AssertionError(
            f"{what}: {int(bad.sum())} of {err.size} outside |d| <= {rtol}*|ref| + atol; "
            f"worst at {i}: got {got[i]!r} want {want[i]!r}")
