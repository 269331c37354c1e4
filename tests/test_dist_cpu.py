"""Multi-rank host logic on CPU (gloo, world size 2 and 3).

Each rank takes its shard plan (``ptxc.dist.shard_plan``), computes its shard
with the float64 oracle on the element ranges the plan names (standing in for
the GPU kernel), and the shards are all-gathered; the result must equal the
oracle over the whole tensor.  Split-K across ranks sums per-rank partials with
``reduce_scatter_rows`` (all-reduce + row slice on gloo, reduce-scatter on
NCCL).  No GPU is touched.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from emmy_ir import synth
from oracle import formulas as F
from ptxc import Lowerer
from ptxc.dist import reduce_scatter_rows, shard_plan, shard_ranges, splitk_plan


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _shaped(meta, arrays):
    shp = {a["name"]: a["shape"] for a in meta["args"]}
    return {k: v.reshape(shp[k]) for k, v in arrays.items()}


def _family_result(plan, meta, full):
    """Oracle output of a (possibly sharded) plan from the flat arrays of its shard."""
    fam, a = plan["family"], plan["args"]
    if fam == "softmax":
        v = plan["view"]
        x = full[a["x"]].reshape(v["outer"], v["n"], v["inner"])
        return F.softmax(x, axis=1, out_dtype=np.float64).reshape(-1)
    if fam == "rownorm":
        v = plan["view"]
        x = full[a["x"]].reshape(v["outer"], v["n"])
        eps = [m["data"][0] for m in meta["args"] if m["name"] == a.get("eps")]
        if plan["params"]["mode"] == "layer":
            return F.layernorm(x, full.get(a.get("w")), full.get(a.get("b")), eps[0],
                               out_dtype=np.float64).reshape(-1)
        return F.rmsnorm(x, full.get(a.get("w")), eps[0], out_dtype=np.float64).reshape(-1)
    if fam == "reduce":
        v = plan["view"]
        x = full[a["x"]].reshape(v["outer"], v["n"], v["inner"])
        op = "mean" if plan["params"]["mean"] else plan["params"]["op"]
        return np.asarray(F.reduce(x, 1, op, out_dtype=np.float64)).reshape(-1)
    if fam.startswith("gemm"):
        g = plan["gemm"]
        A = full[a["a"]].reshape(g["batch"], g["m"], g["k"])
        B = full[a["b"]].reshape(g["batch"], g["k"], g["n"])
        bias = full.get(a.get("bias"))
        return F.matmul(A, B, bias if (g["epilogue"] & 1) else None, bool(g["epilogue"] & 2),
                        out_dtype=np.float64).reshape(-1)
    if fam.startswith("attention"):
        g = plan["attention"]
        q = full[a["q"]].reshape(1, g["batch"], g["sq"], g["d"])
        k = full[a["k"]].reshape(1, g["batch"], g["sk"], g["d"])
        vv = full[a["v"]].reshape(1, g["batch"], g["sk"], g["dv"])
        div = [m["data"][0] for m in meta["args"] if m["name"] == a["scale"]][0]
        return F.attention_bhsd(q, k, vv, 1.0 / div, out_dtype=np.float64).reshape(-1)
    if fam == "pointwise":
        # float64 walk of the plan's register program (add / multiply only here)
        g = plan["pointwise"]
        regs = [full[n] for n in g["inputs"]] + [full[n] for n in g["scalars"]] + \
            [np.float64(v) for v in g["immediates"]]
        for op, _dst, ra, rb, _rc in g["program"]:
            x, y = regs[ra], regs[rb]
            regs.append({1: lambda: x + y, 3: lambda: x * y}[op]())
        return np.asarray(regs[g["result_reg"]], dtype=np.float64).reshape(-1)
    if fam == "pointwise_int":
        # s64 walk of the integer program (add / multiply only here), wrapping
        g = plan["pointwise"]
        regs = [full[n].astype(np.int64).view(np.uint64) for n in g["inputs"]] + \
            [full[n].astype(np.int64).view(np.uint64) for n in g["scalars"]] + \
            [np.array(v, np.int64).view(np.uint64) for v in g["immediates"]]
        for op, _dst, ra, rb, _rc in g["program"]:
            x, y = regs[ra], regs[rb]
            regs.append({1: lambda: x + y, 3: lambda: x * y}[op]())
        return np.asarray(regs[g["result_reg"]]).view(np.int64).astype(np.float64).reshape(-1)
    raise ValueError(fam)


CASES = {
    "softmax": lambda: synth.softmax([6, 5, 64]),
    "softmax_dim0": lambda: synth.softmax([40, 7], dim=0),
    "layernorm": lambda: synth.layernorm(11, 96),
    "rmsnorm": lambda: synth.rmsnorm(9, 64),
    "reduce_mid": lambda: synth.reduce([5, 12, 8], 1, "mean"),
    "gemm_rows": lambda: synth.matmul(96, 64, 32, bias=True, relu=True, tm=32, tn=32),
    "bmm_batches": lambda: synth.matmul(32, 32, 16, batch=5, tm=32, tn=32),
    "attention_heads": lambda: synth.attention(2, 3, 16, 16, dtype="f32"),
    "pointwise_elements": lambda: synth.pointwise(
        1001, ("add", ("multiply", ("const", "c", 1.5), "x0"), "x1"), "f32"),
    "pointwise_int_elements": lambda: synth.pointwise(
        1001, ("add", ("multiply", ("const", "c", 3), "x0"), "x1"), "i32",
        inits={"x0": {"dist": "int", "low": -1000, "high": 1000},
               "x1": {"dist": "int", "low": -1000, "high": 1000}}),
}


def _worker(rank, world, port, case, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        kop, meta = CASES[case]()
        plan = Lowerer(kop, meta).plan()
        host = synth.make_inputs(meta)
        sub, slices = shard_plan(plan, rank, world)
        local = {}
        for name, (off, cnt) in slices.items():
            local[name] = host[name][off:off + cnt]
        for name in sub.get("pointwise", {}).get("scalars", []):
            local[name] = host[name]
        out_name = plan["outputs"][0]
        mine = _family_result(sub, meta, local)
        pieces = [None] * world
        dist.all_gather_object(pieces, mine)
        if rank == 0:
            got = np.concatenate(pieces)
            want = _family_result(plan, meta, host)
            q.put((got.shape == want.shape) and bool(np.allclose(got, want, rtol=1e-12, atol=1e-12)))
    finally:
        dist.destroy_process_group()


def _splitk_worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        kop, meta = synth.matmul(64, 32, 96, splits=8, tm=32, tn=32, bk=4)
        plan = Lowerer(kop, meta).plan()
        host = _shaped(meta, synth.make_inputs(meta))
        sub, slices, (k0, k1) = splitk_plan(plan, rank, world)
        A = host["A"][:, k0:k1].astype(np.float64)
        B = host["B"][k0:k1].astype(np.float64)
        assert sub["gemm"]["k"] == k1 - k0
        partial = torch.from_numpy(A @ B)
        rows = reduce_scatter_rows(partial)
        pieces = [torch.zeros_like(rows) for _ in range(world)]
        dist.all_gather(pieces, rows)
        if rank == 0:
            got = torch.cat(pieces).numpy()
            want = host["A"].astype(np.float64) @ host["B"].astype(np.float64)
            q.put(bool(np.allclose(got, want, rtol=1e-12, atol=1e-12)))
    finally:
        dist.destroy_process_group()


def _spawn(fn, world, *args):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=fn, args=(r, world, port) + args + (q,)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    codes = [p.exitcode for p in procs]
    for p in procs:
        if p.is_alive():
            p.kill()
    assert codes == [0] * world, codes
    return q.get(timeout=5)


@pytest.mark.parametrize("case", sorted(CASES))
def test_sharded_plans_reassemble_the_full_result(case):
    assert _spawn(_worker, 2, case)


def test_three_ranks_uneven_rows():
    assert _spawn(_worker, 3, "layernorm")


def test_splitk_across_ranks_reduce_scatters_the_sum():
    assert _spawn(_splitk_worker, 2)


def test_shard_ranges_cover_exactly_once():
    for n in (0, 1, 7, 100, 257):
        for w in (1, 2, 3, 8):
            r = shard_ranges(n, w)
            assert r[0][0] == 0 and r[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(r, r[1:]))
            assert max(e - s for s, e in r) - min(e - s for s, e in r) <= 1


@pytest.mark.parametrize("world", [2, 4, 8])
def test_every_bench_configuration_shards(world):
    """The per-family bench key at N > 1 times each rank's ``shard_plan`` shard:
    every configuration it names has one, and the shards of each sliced tensor
    cover it exactly once."""
    import math
    import bench
    for name, (kop, meta) in bench.family_cases().items():
        if name.startswith(("K4a", "K5_sweep")):
            continue
        plan = Lowerer(kop, meta).plan()
        covered = {}
        for rank in range(world):
            sub, slices = shard_plan(plan, rank, world)
            assert sub["shard"] == {"rank": rank, "world": world}
            for t, (off, cnt) in slices.items():
                covered.setdefault(t, []).append((off, cnt))
        for t, parts in covered.items():
            full = math.prod(plan["tensors"][t]["shape"])
            if all(p == (0, full) for p in parts):
                continue                                  # replicated on every rank
            parts.sort()
            assert parts[0][0] == 0, (name, t)
            assert all(a[0] + a[1] == b[0] for a, b in zip(parts, parts[1:])), (name, t)
            assert parts[-1][0] + parts[-1][1] == full, (name, t)


def test_roofline_over_several_gpus_scales_every_peak():
    """The per-family roofline at N > 1: every peak is N times the single-GPU
    one, so the fraction of a time that scales as 1/N stays the same."""
    import bench
    nbytes, us = 1 << 30, 200.0
    one = bench.roofline_block("K2a_softmax_32x16x512x512", nbytes, 0.0, us, None)
    four = bench.roofline_block("K2a_softmax_32x16x512x512", nbytes, 0.0, us / 4, None, gpus=4)
    assert four["bound"] == one["bound"] == "hbm"
    assert abs(four["peak"] - 4 * one["peak"]) < 0.5
    assert abs(four["frac"] - one["frac"]) < 1e-3
    assert four["traffic"] is None and four["peak_source"].endswith("x 4 GPUs")
    flops = 2.0 * 4096 * 8192 * 2048
    t1 = bench.roofline_block("K3a_gemm_f16_4096x2048x8192_bias_relu", 117_440_512, flops, 110.0,
                              "tensor")
    t2 = bench.roofline_block("K3a_gemm_f16_4096x2048x8192_bias_relu", 117_440_512, flops, 55.0,
                              "tensor", gpus=2)
    assert t1["bound"] == t2["bound"] == "tensor"
    assert abs(t2["frac"] - t1["frac"]) < 1e-3
    att = bench.roofline_block("K5", 1 << 27, 1.0, 30.0, "tensor", n_exp=1 << 40, gpus=2)
    assert att["bound"] == "mufu" and abs(att["peak"] - 2 * bench.MUFU_EXP_PER_S / 1e12) < 1e-3
