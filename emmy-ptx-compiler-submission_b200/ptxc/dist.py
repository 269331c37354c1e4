"""Sharding launch plans over the GPUs of one node (one process per GPU).

The kernel families split along independent units, so a shard is just a
smaller plan over a contiguous slice of each tensor and needs no collective on
the data path:

* reduce / rownorm / softmax / matvec: rows of the ``[outer, n, inner]`` view
  (x and y sliced by rows; weights, bias and scalar constants replicated);
* matmul (f32 and f16): batches when there are at least as many as ranks,
  otherwise rows of A and C (B and the bias replicated);
* attention: (batch, head) slices of q, k, v and o;
* pointwise: contiguous element ranges of every input and the output (the
  one-element constant tensors and broadcast inputs replicated; the shard's
  first element index keeps the broadcast reads in place).

The one family with an exchange step is split-K matmul spread over ranks:
each rank multiplies its K slice into a full-size partial C, and the partials
are summed with a reduce-scatter (NCCL over NVLink on GPUs), leaving each rank
its rows of C -- the multi-GPU form of the reference's atomic split-K writes
(``ptxc/stmts.py:456-461``).

``shard_plan`` returns the rank's plan plus, per tensor, the element range of
the full tensor it covers; ``ptxc.launch.run`` runs it unchanged.
"""

from __future__ import annotations

import copy
import math


def shard_ranges(n: int, world: int) -> list:
    """Balanced contiguous ranges ``[(start, stop), ...]`` of ``n`` units over ``world`` ranks."""
    base, extra = divmod(n, world)
    out, s = [], 0
    for r in range(world):
        e = s + base + (1 if r < extra else 0)
        out.append((s, e))
        s = e
    return out


def _numel(shape):
    return math.prod(shape) if shape else 1


def shard_plan(plan: dict, rank: int, world: int):
    """This rank's plan and ``{tensor: (element offset, element count)}`` into the full tensors."""
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world {world}")
    sub = copy.deepcopy(plan)
    fam = plan["family"]
    a = plan["args"]
    slices = {name: (0, _numel(spec["shape"])) for name, spec in plan["tensors"].items()}

    def set_shape(name, shape):
        sub["tensors"][name]["shape"] = list(shape)

    if fam in ("reduce", "rownorm", "softmax", "matvec", "rowop"):
        v = plan["view"]
        lo, hi = shard_ranges(v["outer"], world)[rank]
        rows = hi - lo
        sub["view"]["outer"] = rows
        x_row = v["n"] * v["inner"]
        reduces = fam in ("reduce", "matvec") or (
            fam == "rowop" and plan["params"]["mode"] in ("sum", "max", "min", "dot"))
        y_row = v["inner"] if reduces else x_row
        slices[a["x"]] = (lo * x_row, rows * x_row)
        slices[a["y"]] = (lo * y_row, rows * y_row)
        set_shape(a["x"], [rows, v["n"], v["inner"]] if v["inner"] > 1 else [rows, v["n"]])
        set_shape(a["y"], ([rows, v["inner"]] if v["inner"] > 1 else [rows])
                  if reduces else
                  ([rows, v["n"], v["inner"]] if v["inner"] > 1 else [rows, v["n"]]))
    elif fam in ("gemm_f32", "gemm_f64", "gemm_f16"):
        g = plan["gemm"]
        if g["batch"] >= world:
            lo, hi = shard_ranges(g["batch"], world)[rank]
            sub["gemm"]["batch"] = hi - lo
            for role, bstride in (("a", g["a_batch_stride"]), ("b", g["b_batch_stride"]),
                                  ("c", g["c_batch_stride"])):
                slices[a[role]] = (lo * bstride, (hi - lo) * bstride)
            set_shape(a["a"], [hi - lo, g["m"], g["k"]])
            set_shape(a["b"], [hi - lo, g["k"], g["n"]])
            set_shape(a["c"], [hi - lo, g["m"], g["n"]])
        else:
            if g["batch"] != 1:
                raise ValueError("row sharding of a batched matmul with fewer batches than ranks")
            lo, hi = shard_ranges(g["m"], world)[rank]
            rows = hi - lo
            sub["gemm"]["m"] = rows
            sub["gemm"]["a_batch_stride"] = rows * g["k"]
            sub["gemm"]["c_batch_stride"] = rows * g["n"]
            slices[a["a"]] = (lo * g["k"], rows * g["k"])
            slices[a["c"]] = (lo * g["n"], rows * g["n"])
            set_shape(a["a"], [rows, g["k"]])
            set_shape(a["c"], [rows, g["n"]])
    elif fam in ("attention_f32", "attention_f16"):
        g = plan["attention"]
        lo, hi = shard_ranges(g["batch"], world)[rank]
        sub["attention"]["batch"] = hi - lo
        per = {"q": g["sq"] * g["d"], "k": g["sk"] * g["d"], "v": g["sk"] * g["dv"],
               "o": g["sq"] * g["dv"]}
        for role, size in per.items():
            slices[a[role]] = (lo * size, (hi - lo) * size)
        set_shape(a["q"], [hi - lo, g["sq"], g["d"]])
        set_shape(a["k"], [hi - lo, g["d"], g["sk"]] if g["k_transposed"] else [hi - lo, g["sk"], g["d"]])
        set_shape(a["v"], [hi - lo, g["sk"], g["dv"]])
        set_shape(a["o"], [hi - lo, g["sq"], g["dv"]])
    elif fam == "pointwise":
        g = plan["pointwise"]
        lo, hi = shard_ranges(g["n"], world)[rank]
        sub["pointwise"]["n"] = hi - lo
        index = g.get("input_index") or [[0, 0]] * len(g["inputs"])
        bcast = {n for n, (d, _) in zip(g["inputs"], index) if d}
        if bcast & ({n for n, (d, _) in zip(g["inputs"], index) if not d} | {a["out"]}):
            raise ValueError("a pointwise tensor read both whole and broadcast")
        if bcast:
            # broadcast inputs stay whole; the shard numbers its elements from lo
            sub["pointwise"]["first"] = g.get("first", 0) + lo
        for name in list(g["inputs"]) + [a["out"]]:
            if name not in bcast:
                slices[name] = (lo, hi - lo)
                set_shape(name, [hi - lo])
    else:
        raise ValueError(f"family {fam!r} has no sharding rule")
    sub["shard"] = {"rank": rank, "world": world}
    return sub, slices


def splitk_plan(plan: dict, rank: int, world: int):
    """This rank's part of a matmul split along K across ranks.

    Returns (plan, slices, k_range): the rank multiplies A[:, k0:k1] @ B[k0:k1, :]
    into a full-size partial C (its own buffer); ``reduce_scatter_rows`` then
    sums the partials and leaves each rank its rows of C.  ``slices`` gives the
    rows of B the rank reads (A's K slice is strided: the caller passes
    A[:, k0:k1] as its own contiguous tensor).
    """
    if plan["family"] not in ("gemm_f32", "gemm_f64", "gemm_f16"):
        raise ValueError("split-K sharding applies to matmul plans")
    g = plan["gemm"]
    if g["batch"] != 1:
        raise ValueError("split-K sharding of a batched matmul is not supported")
    k0, k1 = shard_ranges(g["k"], world)[rank]
    sub = copy.deepcopy(plan)
    a = plan["args"]
    kk = k1 - k0
    sub["gemm"]["k"] = kk
    sub["gemm"]["a_batch_stride"] = g["m"] * kk
    sub["gemm"]["b_batch_stride"] = kk * g["n"]
    sub["gemm"]["splits"] = max(1, (g["splits"] + world - 1) // world)
    sub["gemm"]["accumulate"] = False
    sub["zero_outputs"] = []
    sub["tensors"][a["a"]]["shape"] = [g["m"], kk]
    sub["tensors"][a["b"]]["shape"] = [kk, g["n"]]
    if "bias" in a and rank != 0:
        # the bias joins the sum once
        sub["gemm"]["epilogue"] = sub["gemm"]["epilogue"] & ~1
    slices = {a["b"]: (k0 * g["n"], kk * g["n"])}
    sub["shard"] = {"rank": rank, "world": world, "split": "k"}
    return sub, slices, (k0, k1)


def reduce_scatter_rows(partial, group=None):
    """Sum a full-size partial ``[M, N]`` over the group and return this rank's rows.

    Uses ``reduce_scatter_tensor`` (NCCL); process groups without it (gloo)
    get the same result from an all-reduce and a row slice.
    """
    import torch
    import torch.distributed as dist
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    M = partial.shape[0]
    lo, hi = shard_ranges(M, world)[rank]
    if M % world == 0 and dist.get_backend(group) == "nccl":
        out = torch.empty((M // world,) + tuple(partial.shape[1:]), dtype=partial.dtype,
                          device=partial.device)
        dist.reduce_scatter_tensor(out, partial.contiguous(), op=dist.ReduceOp.SUM, group=group)
        return out
    full = partial.clone()
    dist.all_reduce(full, op=dist.ReduceOp.SUM, group=group)
    return full[lo:hi].contiguous()
