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
    elif fam in ("pointwise", "pointwise_int"):
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


class PeerRows:
    """Every rank's slot buffer, mapped into this rank's address space.

    Each rank owns ``slots``, a CUDA tensor ``[world, M / world, N]``: slot r
    receives rank r's partial sums of the rows this rank owns.  The buffers
    are exchanged as CUDA IPC handles (``emmy_ipc_export`` /
    ``emmy_ipc_import``) so a kernel on any rank can store into any owner's
    slot over NVLink.  ``ptrs`` lists the owners' slot buffers in rank order
    (this rank's own at its index).  ``close()`` unmaps the peers' buffers;
    call it on every rank before the process group goes away.
    """

    def __init__(self, slots, group=None):
        import ctypes
        import torch.distributed as dist
        from .launch import LibraryError, load_library
        self.lib = load_library()
        self.slots = slots
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        if slots.dim() != 3 or slots.shape[0] != self.world or not slots.is_contiguous():
            raise ValueError("slots must be a contiguous [world, rows per rank, N] tensor")
        handle = (ctypes.c_ubyte * 64)()
        offset = ctypes.c_int64()
        rc = self.lib.emmy_ipc_export(ctypes.c_void_p(slots.data_ptr()), handle,
                                      ctypes.byref(offset))
        if rc:
            raise LibraryError("emmy_ipc_export: " + self.lib.emmy_last_error().decode())
        mine = (bytes(handle), int(offset.value))
        allh = [None] * self.world
        dist.all_gather_object(allh, mine, group=group)
        self.ptrs, self._bases = [], []
        for r, (h, off) in enumerate(allh):
            if r == self.rank:
                self.ptrs.append(slots.data_ptr())
                continue
            hb = (ctypes.c_ubyte * 64).from_buffer_copy(h)
            p, base = ctypes.c_void_p(), ctypes.c_void_p()
            rc = self.lib.emmy_ipc_import(hb, ctypes.c_int64(off), ctypes.byref(p),
                                          ctypes.byref(base))
            if rc:
                self.close()
                raise LibraryError("emmy_ipc_import: " + self.lib.emmy_last_error().decode())
            self.ptrs.append(p.value)
            self._bases.append(base.value)

    def workspace(self, M, N):
        """The local tile workspace and arrival counters (zero; kernels leave them zero)."""
        import torch
        key = (M, N)
        if getattr(self, "_ws_key", None) != key:
            tiles = ((M + 63) // 64) * ((N + 63) // 64)
            self._ws = torch.zeros(M * N, dtype=torch.float32, device=self.slots.device)
            self._counters = torch.zeros(tiles, dtype=torch.int32, device=self.slots.device)
            self._ws_key = key
        return self._ws, self._counters

    def close(self):
        import ctypes
        for b in self._bases:
            self.lib.emmy_ipc_close(ctypes.c_void_p(b))
        self._bases = []


def splitk_to_peers(a_slice, b_slice, peers, M, N, splits=0, bias=None, stream=None):
    """This rank's K slice of ``A @ B``, its rows stored straight into their
    owners' slots: the matmul and the scatter of its partial sums in one
    kernel (``emmy_gemm_f32_rows_to_peers``; rows of other owners travel over
    NVLink as plain 16-byte stores, no partial C is stored locally).

    Every rank's previous sums must be done reading the slots before any rank
    launches, and every rank's launch must be finished before an owner sums
    its slots: ``splitk_step`` does both.
    """
    import ctypes
    import torch
    from .launch import _check, _stream_handle
    lib = peers.lib
    world = peers.world
    ptrs = (ctypes.c_void_p * 8)(*([ctypes.c_void_p(p) for p in peers.ptrs] +
                                   [ctypes.c_void_p(0)] * (8 - world)))
    ws, counters = peers.workspace(M, N)
    st = stream if stream is not None else torch.cuda.current_stream()
    _check(lib.emmy_gemm_f32_rows_to_peers(
        ctypes.c_void_p(a_slice.data_ptr()), ctypes.c_void_p(b_slice.data_ptr()),
        ctypes.c_void_p(bias.data_ptr()) if bias is not None else None, ptrs,
        peers.slots.numel(), world, peers.rank, M // world, M, N, a_slice.shape[-1], splits, ctypes.c_void_p(ws.data_ptr()),
        ctypes.c_void_p(counters.data_ptr()), counters.numel(), _stream_handle(st)),
        "emmy_gemm_f32_rows_to_peers")


def sum_slots(peers, out=None, stream=None):
    """This rank's rows: the sum of its ``world`` slots (``emmy_reduce_f32``
    over the slot axis of the ``[world, rows * N]`` view)."""
    import ctypes
    import torch
    from .launch import _check, _stream_handle
    world, rows, N = peers.slots.shape
    if out is None:
        out = torch.empty(rows, N, dtype=torch.float32, device=peers.slots.device)
    st = stream if stream is not None else torch.cuda.current_stream()
    _check(peers.lib.emmy_reduce_f32(ctypes.c_void_p(peers.slots.data_ptr()),
                                     ctypes.c_void_p(out.data_ptr()), 1, world, rows * N, 0, 0,
                                     None, None, 0, _stream_handle(st)), "emmy_reduce_f32")
    return out


def splitk_step(a_slice, b_slice, peers, M, N, splits=0, bias=None, out=None):
    """One fused split-K step: wait for every rank (the slots are free), launch
    ``splitk_to_peers``, wait for every rank (the slots are full), sum this
    rank's slots.  Returns this rank's rows of ``A @ B``."""
    import torch
    import torch.distributed as dist
    torch.cuda.synchronize()
    dist.barrier(group=peers.group)
    splitk_to_peers(a_slice, b_slice, peers, M, N, splits, bias)
    torch.cuda.synchronize()
    dist.barrier(group=peers.group)
    return sum_slots(peers, out)


class PeerPartials:
    """Every rank's double-buffered split-K partials and flag words, mapped
    into this rank's address space (CUDA IPC, as ``PeerRows``).

    Each rank owns ``parts``, a CUDA tensor ``[2, M, N]`` (step s writes
    buffer ``s % 2``), and ``flags``, ``world`` int64 words that the other
    ranks set to the step they have finished.  ``emmy_peer_reduce_rows``
    reads every rank's buffer of the step for this rank's rows once all flags
    show the step (``splitk_pull_step``).  ``close()`` unmaps the peers'
    buffers; call it on every rank before the process group goes away.
    """

    def __init__(self, M, N, device, group=None):
        import ctypes
        import torch
        import torch.distributed as dist
        from .launch import LibraryError, load_library
        self.lib = load_library()
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.M, self.N = M, N
        self.parts = torch.zeros(2, M, N, dtype=torch.float32, device=device)
        self.flags = torch.zeros(self.world, dtype=torch.int64, device=device)
        self.seq = 0
        mine = []
        for t in (self.parts, self.flags):
            handle = (ctypes.c_ubyte * 64)()
            offset = ctypes.c_int64()
            rc = self.lib.emmy_ipc_export(ctypes.c_void_p(t.data_ptr()), handle,
                                          ctypes.byref(offset))
            if rc:
                raise LibraryError("emmy_ipc_export: " + self.lib.emmy_last_error().decode())
            mine.append((bytes(handle), int(offset.value)))
        allh = [None] * self.world
        torch.cuda.synchronize(device)
        dist.all_gather_object(allh, mine, group=group)
        self.part_ptrs, self.flag_ptrs, self._bases = [], [], []
        for r, handles in enumerate(allh):
            if r == self.rank:
                self.part_ptrs.append(self.parts.data_ptr())
                self.flag_ptrs.append(self.flags.data_ptr())
                continue
            got = []
            for h, off in handles:
                hb = (ctypes.c_ubyte * 64).from_buffer_copy(h)
                p, base = ctypes.c_void_p(), ctypes.c_void_p()
                rc = self.lib.emmy_ipc_import(hb, ctypes.c_int64(off), ctypes.byref(p),
                                              ctypes.byref(base))
                if rc:
                    self.close()
                    raise LibraryError("emmy_ipc_import: " + self.lib.emmy_last_error().decode())
                got.append(p.value)
                self._bases.append(base.value)
            self.part_ptrs.append(got[0])
            self.flag_ptrs.append(got[1])

    def close(self):
        import ctypes
        for b in self._bases:
            self.lib.emmy_ipc_close(ctypes.c_void_p(b))
        self._bases = []


def splitk_pull_gemm(a_slice, b_slice, peers, splits=0, bias=None, stream=None):
    """The first half of ``splitk_pull_step``: start the next step and run this
    rank's K slice into its partial buffer of the step (the f32 GEMM with
    in-GPU atomic split-K; the bias on rank 0 only)."""
    import ctypes
    import torch
    from .launch import _check, _stream_handle
    lib = peers.lib
    M, N, rank = peers.M, peers.N, peers.rank
    K = a_slice.shape[-1]
    st = stream if stream is not None else torch.cuda.current_stream()
    peers.seq += 1
    c = peers.parts[peers.seq % 2]
    use_bias = bias is not None and rank == 0
    _check(lib.emmy_gemm_f32(ctypes.c_void_p(a_slice.data_ptr()), ctypes.c_void_p(b_slice.data_ptr()),
                             ctypes.c_void_p(bias.data_ptr()) if use_bias else None,
                             ctypes.c_void_p(c.data_ptr()), 1, M, N, K, 0, 0, 0, splits, 0,
                             1 if use_bias else 0, _stream_handle(st)), "emmy_gemm_f32")


def splitk_pull_reduce(peers, out=None, stream=None):
    """The second half: ``emmy_peer_reduce_rows`` publishes the step, waits for
    every rank's, and sums every rank's partial of this rank's rows."""
    import ctypes
    import torch
    from .launch import _check, _stream_handle
    lib = peers.lib
    M, N, world, rank = peers.M, peers.N, peers.world, peers.rank
    st = stream if stream is not None else torch.cuda.current_stream()
    buf = peers.seq % 2
    c = peers.parts[buf]
    lo, hi = shard_ranges(M, world)[rank]
    if out is None:
        out = torch.empty(hi - lo, N, dtype=torch.float32, device=c.device)
    off = buf * M * N * 4
    parts = (ctypes.c_void_p * world)(*[ctypes.c_void_p(p + off) for p in peers.part_ptrs])
    flags = (ctypes.c_void_p * world)(*[ctypes.c_void_p(p) for p in peers.flag_ptrs])
    _check(lib.emmy_peer_reduce_rows(parts, flags, world, rank, peers.seq, lo, hi - lo, N,
                                     ctypes.c_void_p(out.data_ptr()), _stream_handle(st)),
           "emmy_peer_reduce_rows")
    return out


def splitk_pull_step(a_slice, b_slice, peers, splits=0, bias=None, out=None, stream=None):
    """One split-K step with the exchange over peer memory, no host barrier:
    ``splitk_pull_gemm`` then ``splitk_pull_reduce``.  Returns this rank's
    rows of ``A @ B`` (+ bias), ``[rows, N]``."""
    splitk_pull_gemm(a_slice, b_slice, peers, splits, bias, stream)
    return splitk_pull_reduce(peers, out, stream)
