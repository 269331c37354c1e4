"""Multi-GPU paths on 2 GPUs of one node (skipped with fewer).

* sharded plans: each rank runs its row shard of a softmax and its (batch,
  head) shard of the tcgen05 attention through the C ABI on its own GPU; the
  shards are all-gathered over NCCL and compared with the float64 oracle;
* split-K across GPUs: each rank multiplies its K slice with the f32 GEMM into
  a full partial C, and ``reduce_scatter_rows`` sums the partials over NCCL;
  then the fused form: the GEMM stores its partial rows straight into their
  owner's slot over NVLink and each owner sums its slots (``PeerRows`` +
  ``splitk_step``); then the exchange over peer memory with no host
  barrier (``PeerPartials`` + ``splitk_pull_step``: step flags in each
  rank's memory, bounded waits, double-buffered partials; three steps).

Tolerances as in the single-GPU tests (``tests/parity.py``): softmax 1e-5
relative, attention 1e-3 of ``sum_j p_j |v_j|``, split-K 1e-5 of ``|A| @ |B|``.  NVLS is off (``NCCL_NVLS_ENABLE=0``).
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _gpus():
    import torch
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, q):
    import sys
    from datetime import timedelta
    from pathlib import Path
    root = Path(__file__).resolve().parent.parent
    for p in (str(root), str(root / "emmy-ptx-compiler-submission_b200")):
        sys.path.insert(0, p)
    # NVLS off; NCCL's communicator set-up (ranks, devices) logged to stderr
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0",
                      NCCL_DEBUG="INFO", NCCL_DEBUG_SUBSYS="INIT", NCCL_DEBUG_FILE="/dev/stderr")
    import torch
    import torch.distributed as dist
    from emmy_ir import synth
    from oracle import formulas as F
    from ptxc import Lowerer
    from ptxc.dist import (PeerPartials, PeerRows, reduce_scatter_rows, shard_plan, splitk_plan,
                           splitk_pull_step, splitk_step)
    from ptxc.launch import Executor, load_library
    import ctypes
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    ok = True
    try:
        # --- softmax rows, sharded
        kop, meta = synth.softmax([64, 1024], x_init={"dist": "normal", "std": 2.0})
        plan = Lowerer(kop, meta).plan()
        host = synth.make_inputs(meta)
        sub, slices = shard_plan(plan, rank, world)
        ex = Executor(sub)
        ex.upload({n: host[n][o:o + c] for n, (o, c) in slices.items()})
        ex.launch()
        mine = ex.tensors["y"]
        out = torch.empty(64 * 1024, device="cuda")
        dist.all_gather_into_tensor(out, mine)
        if rank == 0:
            ref = F.softmax(host["x"].reshape(64, 1024), out_dtype=np.float64).reshape(-1)
            got = out.cpu().numpy().astype(np.float64)
            ok &= bool(np.all(np.abs(got - ref) <= 1e-5 * np.abs(ref) + 1e-30))
        # --- attention heads, sharded (tcgen05 path)
        kop, meta = synth.attention(2, 4, 256, 128, dtype="f16", out_dtype="f32")
        plan = Lowerer(kop, meta).plan()
        host = synth.make_inputs(meta)
        sub, slices = shard_plan(plan, rank, world)
        ex = Executor(sub)
        ex.upload({n: host[n][o:o + c] for n, (o, c) in slices.items() if n in host})
        ex.launch()
        out = torch.empty(2 * 4 * 256 * 128, device="cuda")
        dist.all_gather_into_tensor(out, ex.tensors["o"])
        if rank == 0:
            x = {k: v.reshape(2, 4, 256, 128) for k, v in host.items() if v.size > 1}
            ref = F.attention_bhsd(x["q"], x["k"], x["v"], 1 / np.sqrt(128), out_dtype=np.float64)
            scale = F.attention_abs_scale(x["q"], x["k"], x["v"], 1 / np.sqrt(128))
            got = out.cpu().numpy().astype(np.float64).reshape(ref.shape)
            ok &= bool(np.all(np.abs(got - ref) <= 1e-3 * scale))
        # --- split-K f32 GEMM across ranks + NCCL reduce-scatter
        kop, meta = synth.matmul(256, 256, 8192, splits=16, tm=128, tn=128, rm=8, rn=8)
        plan = Lowerer(kop, meta).plan()
        host = synth.make_inputs(meta)
        A = host["A"].reshape(256, 8192)
        B = host["B"].reshape(8192, 256)
        sub, slices, (k0, k1) = splitk_plan(plan, rank, world)
        a_loc = torch.from_numpy(np.ascontiguousarray(A[:, k0:k1])).cuda()
        b_loc = torch.from_numpy(np.ascontiguousarray(B[k0:k1])).cuda()
        c_part = torch.empty(256, 256, device="cuda")
        lib = load_library()
        P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
        g = sub["gemm"]
        rc = lib.emmy_gemm_f32(P(a_loc), P(b_loc), None, P(c_part), 1, 256, 256, g["k"], 0, 0, 0,
                               g["splits"], 0, 0, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        assert rc == 0
        rows = reduce_scatter_rows(c_part)
        full = torch.empty(256, 256, device="cuda")
        dist.all_gather_into_tensor(full, rows)
        if rank == 0:
            ref = A.astype(np.float64) @ B.astype(np.float64)
            scale = np.abs(A).astype(np.float64) @ np.abs(B).astype(np.float64)
            ok &= bool(np.all(np.abs(full.cpu().numpy() - ref) <= 1e-5 * scale))
        # --- the same split-K with the reduce-scatter fused into the GEMM:
        # partial rows go straight into their owner's buffer over NVLink
        slots = torch.full((world, 256 // world, 256), float("nan"), device="cuda")
        peers = PeerRows(slots)
        try:
            for _ in range(2):                     # twice: the workspace is left clean
                mine = splitk_step(a_loc, b_loc, peers, 256, 256, splits=g["splits"])
            full2 = torch.empty(256, 256, device="cuda")
            dist.all_gather_into_tensor(full2, mine)
            if rank == 0:
                ok &= bool(np.all(np.abs(full2.cpu().numpy() - ref) <= 1e-5 * scale))
        finally:
            torch.cuda.synchronize()
            dist.barrier()
            peers.close()
        # --- the exchange over peer memory with no host barrier: each rank's
        # partial into its buffer of the step, then every rank sums its rows
        # of every partial once all have published the step.  Three steps in
        # a row (both buffers and the step flags turn over), a bias on rank 0.
        bias = torch.linspace(-1.0, 1.0, 256, device="cuda")
        pp = PeerPartials(256, 256, torch.device("cuda"))
        try:
            for _ in range(3):
                mine3 = splitk_pull_step(a_loc, b_loc, pp, splits=g["splits"], bias=bias)
            torch.cuda.synchronize()
            code = ctypes.c_int(0)
            lib.emmy_get_device_status(ctypes.byref(code), None)
            ok &= code.value == 0
            full3 = torch.empty(256, 256, device="cuda")
            dist.all_gather_into_tensor(full3, mine3)
            if rank == 0:
                refb = ref + bias.double().cpu().numpy()
                scaleb = scale + np.abs(bias.double().cpu().numpy())
                ok &= bool(np.all(np.abs(full3.cpu().numpy() - refb) <= 1e-5 * scaleb))
        finally:
            torch.cuda.synchronize()
            dist.barrier()
            pp.close()
        torch.cuda.synchronize()
    finally:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        q.put(ok)


@pytest.mark.skipif(_gpus() < 2, reason="needs 2 GPUs")
def test_two_gpu_shards_and_splitk_reduce_scatter():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    codes = [p.exitcode for p in procs]
    for p in procs:
        if p.is_alive():
            p.kill()
    assert codes == [0, 0], codes
    assert q.get(timeout=5)
