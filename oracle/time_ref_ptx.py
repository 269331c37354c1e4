"""Time the reference compiler's own PTX beside the B200 kernels (test infrastructure).

For each benchmark configuration with PTX in ``oracle/_ref`` (made by
``make_ref_ptx.py``), both sides are timed with the bench's protocol: inputs
resident, a 256 MiB write + 256 MiB read between launches (clean L2), a device
spin before the start event, CUDA events on the launching stream, median of
``--reps``.  The reference side is the unmodified reference PTX launched as its
harness does (``oracle/ref_ptx.py``); outputs that the plan zeroes before
atomic writes are zeroed inside both timed regions.  Prints one JSON line per
configuration.

Usage (on a GPU box): ``python oracle/time_ref_ptx.py [--reps 10]``.
"""

from __future__ import annotations

import argparse
import json
import statistics
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
for p in (str(ROOT), str(ROOT / "emmy-ptx-compiler-submission_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)


def _time(fn, flush, reps, spin):
    import torch
    for _ in range(3):
        fn()
    out = []
    for _ in range(reps):
        flush()
        torch.cuda._sleep(spin)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        fn()
        e1.record()
        e1.synchronize()
        out.append(e0.elapsed_time(e1) * 1e3)
    return statistics.median(out)


def main() -> int:
    import torch
    import bench
    from emmy_ir import synth
    from oracle import ref_ptx
    from oracle.make_ref_ptx import BENCH_CASES
    from ptxc import Lowerer
    from ptxc.launch import Executor
    ap = argparse.ArgumentParser()
    ap.add_argument("--reps", type=int, default=10)
    args = ap.parse_args()
    dev = torch.device("cuda:0")
    torch.cuda.set_device(dev)
    flush = bench.L2Flush(dev)
    for name, make in BENCH_CASES.items():
        if not ref_ptx.available(name):
            continue
        kop, meta = make(synth)
        plan = Lowerer(kop, meta).plan()
        ex = Executor(plan, device=dev)
        for t in ex.tensors.values():
            if t.is_floating_point():
                t.normal_()
        for a in meta["args"]:
            if "data" in a:
                ex.tensors[a["name"]].fill_(float(a["data"][0]))
        ours = _time(ex.launch, flush, args.reps, bench.SPIN_CYCLES)
        k = ref_ptx.RefKernel(name)
        rt = {a["name"]: ex.tensors[a["name"]] for a in meta["args"]}
        zero = [rt[n] for n in plan.get("zero_outputs", [])]

        def ref_launch():
            for z in zero:
                z.zero_()
            k.launch(rt)
        ref = _time(ref_launch, flush, args.reps, bench.SPIN_CYCLES)
        k.close()
        nbytes = bench.plan_bytes(plan)
        line = {"config": name, "family": plan["family"], "b200_us": round(ours, 2),
                "reference_ptx_us": round(ref, 2), "speedup": round(ref / ours, 2),
                "b200_gbs": round(nbytes / ours / 1e3, 1),
                "reference_ptx_gbs": round(nbytes / ref / 1e3, 1)}
        if "gemm" in plan or "attention" in plan:
            if "gemm" in plan:
                g = plan["gemm"]
                flops = 2.0 * g["batch"] * g["m"] * g["n"] * g["k"]
            else:
                g = plan["attention"]
                flops = 2.0 * g["batch"] * g["sq"] * g["sk"] * (g["d"] + g["dv"])
            line["b200_tflops"] = round(flops / ours / 1e6, 2)
            line["reference_ptx_tflops"] = round(flops / ref / 1e6, 2)
        print(json.dumps(line), flush=True)
        del ex
        torch.cuda.empty_cache()
    return 0


if __name__ == "__main__":
    sys.exit(main())
