"""Family matcher for the tiled matmul / batched / split-K IR shape.

Shape (reference fixtures ``v_m_*``, ``w_m_*``; lowering in
``ptxc/stmts.py:1590-1623`` (CpAsyncCopy), ``:663-725`` (Loop), ``:614-632``
(fused multiply-accumulate), ``:434-487`` (Write, atomic ``red.global.add``)):

    Tile([_aS_ks,] [batch,] m-block, n-block, m-lane, n-lane)
      Init acc...                       -- register micro-tile seeds
      Smem _a_smem, _b_smem              -- staging buffers
      [CpAsyncCopy ... prologue]
      StridedLoop _ks over K { CpAsyncCopy A/B tiles; Commit; Wait; Sync;
                               Loop _ki { Load smem A, Load smem B, multiply, Accum add }; Sync }
      [epilogue: Load bias, add, maximum(., 0)]
      Write C[...] (atomic when K is split)

The two staged tensors are told apart by where the inner-loop variable sits in
their shared-memory index (A tile ``[m, k]``, B tile ``[k, n]``); shapes come
from meta.json and must agree (``[b,] M, K`` x ``[b,] K, N`` -> ``[b,] M, N``);
the writes must cover C exactly once per split; the epilogue formula is
probed (``ptxc.scalar``) against none / +bias / relu / +bias then relu.
"""

from __future__ import annotations

import math
import random
import re

from .common import const_int, norm_dtype, op_name, stmt_name
from .match_reduce import NoMatch, need
from .scalar import ProbeMismatch, close, run_scalar

_SPLIT_AXIS = re.compile(r"^_a\d+_ks$")


def _walk(stmts, depth=0):
    for st in stmts:
        yield st, depth
        for attr in ("body", "else_body"):
            child = getattr(st, attr, None)
            if isinstance(child, (tuple, list)) and child:
                yield from _walk(child, depth + 1)


def _uses_var(e, name) -> bool:
    fv = getattr(e, "free_vars", None)
    return bool(fv and name in e.free_vars())


EPILOGUES = {
    0: lambda acc, b: acc,
    1: lambda acc, b: acc + b,
    2: lambda acc, b: max(acc, 0.0),
    3: lambda acc, b: max(acc + b, 0.0),
}


def match_gemm(kop, tile, meta) -> dict:
    shapes, dtypes = meta.shapes, meta.dtypes
    smem = {}
    copies = {}
    for st, _ in _walk(tile.body):
        k = stmt_name(st)
        if k == "Smem":
            smem[st.name] = st
        elif k == "CpAsyncCopy":
            copies.setdefault(st.smem, set()).add(st.src)
    need(len(smem) >= 2 and copies, "no shared-memory staging of two operands")
    need(all(len(v) == 1 for v in copies.values()), "a staging buffer fed from several tensors")
    staged = {s: next(iter(v)) for s, v in copies.items()}
    need(len(staged) == 2 and len(set(staged.values())) == 2, "expected exactly two staged operands")
    for s, src in staged.items():
        need(s in smem and src in shapes, "staging buffer or source unknown")

    # inner product loop(s): a Loop whose body loads both staged buffers
    inner = [st for st, _ in _walk(tile.body) if stmt_name(st) == "Loop"
             and any(stmt_name(s) == "Load" and s.input in staged for s in st.body)]
    need(len(inner) == 1, "no unique inner product loop")
    loop = inner[0]
    ki = loop.axis.name
    loads = {}
    role_of = {}
    accs = set()
    for s in loop.body:
        k = stmt_name(s)
        if k == "Load":
            need(s.input in staged and len(s.names) == 1, "inner loop reads outside the staging buffers")
            idx = tuple(s.index)
            need(len(idx) == 2, "staged operand index is not 2-D")
            if _uses_var(idx[1], ki) and not _uses_var(idx[0], ki):
                role = "a"
            elif _uses_var(idx[0], ki) and not _uses_var(idx[1], ki):
                role = "b"
            else:
                raise NoMatch("inner loop variable position does not tell A from B")
            prev = role_of.get(s.input)
            need(prev in (None, role), "one staging buffer used as both operands")
            role_of[s.input] = role
            loads[s.names[0]] = role
        elif k == "Assign":
            need(op_name(s.op) == "multiply" and len(s.args) == 2, "inner loop op is not a product")
            need(sorted(loads.get(a, "?") for a in s.args) == ["a", "b"], "product is not A x B")
            loads[s.name] = "prod"
        elif k == "Accum":
            need(op_name(s.op) == "add" and s.base is None and loads.get(s.value) == "prod",
                 "inner loop fold is not a sum of products")
            need(norm_dtype(s.dtype) == "f32", "accumulator is not f32")
            accs.add(s.name)
        else:
            raise NoMatch(f"{k} in the inner product loop")
    need(set(role_of.values()) == {"a", "b"}, "inner loop does not read both operands")
    a_name = staged[[s for s, r in role_of.items() if r == "a"][0]]
    b_name = staged[[s for s, r in role_of.items() if r == "b"][0]]

    # statements after the K loop: epilogue and writes (top level of the Tile)
    top = list(tile.body)
    last_loop = max(i for i, s in enumerate(top) if stmt_name(s) in ("StridedLoop", "Loop"))
    tail = top[last_loop + 1:]
    writes = [s for s in tail if stmt_name(s) == "Write"]
    need(writes, "no output writes after the K loop")
    outs = {w.output for w in writes}
    need(len(outs) == 1, "writes to several outputs")
    c_name = outs.pop()
    need(c_name in shapes and c_name not in staged.values(), "output buffer")
    atomic = {bool(w.atomic) for w in writes}
    need(len(atomic) == 1, "mixed atomic and plain writes")
    atomic = atomic.pop()
    bias_name = None
    for s in tail:
        k = stmt_name(s)
        if k == "Load":
            need(len(s.names) == 1 and len(shapes.get(s.input, ())) == 1, "epilogue load is not a vector")
            need(bias_name in (None, s.input), "several epilogue vectors")
            bias_name = s.input
        elif k not in ("Let", "Assign", "Write", "Sync"):
            raise NoMatch(f"{k} after the K loop")

    # probe the epilogue per write
    epilogue = None
    rng = random.Random(7)
    for w in writes:
        need(len(w.values) == 1, "vector output write")
        form = None
        for code, fn in EPILOGUES.items():
            ok = True
            # enough trials that a relu is seen both clipping and passing
            for _ in range(24):
                env = {a: rng.uniform(-3, 3) for a in accs}
                bval = rng.uniform(-2, 2)
                try:
                    run_scalar([s for s in tail if stmt_name(s) != "Write"], env,
                               load=lambda st, bval=bval: [bval])
                    got = env[w.values[0]]
                except (ProbeMismatch, KeyError):
                    ok = False
                    break
                # the write must be this form of one of the accumulators
                cand = [a for a in accs if close(fn(env[a], bval), got)]
                if not cand:
                    ok = False
                    break
            if ok:
                form = code
                break
        need(form is not None, "epilogue is not none / bias / relu / bias+relu")
        need(epilogue in (None, form), "writes use different epilogues")
        epilogue = form
    need((epilogue & 1) == 0 or bias_name is not None, "bias epilogue without a bias vector")
    if atomic:
        need(epilogue == 0, "an epilogue on atomic partial sums is not supported")

    # shapes
    a_shape, b_shape, c_shape = shapes[a_name], shapes[b_name], shapes[c_name]
    need(len(a_shape) == len(b_shape) == len(c_shape) and len(c_shape) in (2, 3), "operand ranks")
    batch = c_shape[0] if len(c_shape) == 3 else 1
    if len(c_shape) == 3:
        need(a_shape[0] == b_shape[0] == batch, "batch sizes differ")
    M, K = a_shape[-2], a_shape[-1]
    K2, N = b_shape[-2], b_shape[-1]
    need(K == K2 and c_shape[-2] == M and c_shape[-1] == N, "operand shapes do not chain")
    if bias_name is not None:
        need(shapes[bias_name] == (N,), "bias is not [N]")

    # coverage: every element of C written once per split
    axes = [(a.name, int(a.extent.value)) for a in tile.axes]
    splits = 1
    for nm, ext in axes:
        if _SPLIT_AXIS.match(nm):
            splits = ext
    lanes = math.prod(e for _, e in axes)
    need(lanes // splits * len(writes) == batch * M * N, "writes do not cover the output exactly")
    if splits > 1:
        need(atomic, "split-K axis without atomic writes")

    adt, bdt, cdt = dtypes[a_name], dtypes[b_name], dtypes[c_name]
    need(adt == bdt, "A and B dtypes differ")
    zero = c_name in meta.zero_outputs
    g = {"batch": batch, "m": M, "n": N, "k": K, "splits": splits,
         "a_batch_stride": M * K, "b_batch_stride": K * N, "c_batch_stride": M * N,
         "accumulate": bool(atomic and not zero), "epilogue": epilogue}
    args = {"a": a_name, "b": b_name, "c": c_name}
    if bias_name is not None:
        args["bias"] = bias_name
    if bias_name is not None:
        need(dtypes[bias_name] == ("f64" if adt == "f64" else "f32"),
             "bias vector dtype (f32, or f64 for an f64 matmul)")
    if adt in ("f32", "f64"):
        need(cdt == adt, f"{adt} matmul with a non-{adt} output")
        return {"family": f"gemm_{adt}", "symbol": f"emmy_gemm_{adt}", "args": args, "gemm": g,
                "params": {}, "dtypes": {"ab": adt, "c": cdt}}
    if adt == "f16":
        need(cdt in ("f32", "f16"), "f16 matmul output must be f16 or f32")
        g["out_dtype"] = 0 if cdt == "f32" else 1
        return {"family": "gemm_f16", "symbol": "emmy_gemm_f16", "args": args, "gemm": g,
                "params": {}, "dtypes": {"ab": adt, "c": cdt}}
    raise NoMatch(f"no B200 matmul kernel for {adt} operands")
