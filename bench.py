#!/usr/bin/env python3
"""Benchmark of the B200 kernel families behind the Emmy Kernel IR drop-in.

Headline workload ("K2"): one step = the softmax IR over
x[32,16,512,512] f32 (dim=-1, x ~ N(0, std 2)) followed by the layernorm IR
over x[16384,1024] f32 (affine, gamma ~ U(0.5,1.5), beta ~ N(0, 0.1),
eps 1e-5).  Both IRs are synthesised in the reduction shapes of the
reference fixtures, compiled to launch plans by ``ptxc.Lowerer`` and run
through the C-ABI of ``libemmyb200.so``.  The metric is HBM throughput over
the algorithmic bytes (every input read once, every output written once).

Arms
  default            the B200 kernels, one process per GPU.  With N ranks the
                     K2 rows are partitioned (``ptxc.dist.shard_plan``): each
                     rank runs 1/N of the softmax rows and 1/N of the layernorm
                     rows, no collective on the data path (strong scaling; the
                     line's ``value`` is the whole workload's bytes over the
                     slowest rank's time).  The ``weak`` key times every rank
                     on a full K2 batch.  At N > 1 the split-K matmul K4a runs
                     across the ranks (each rank a K slice, then the NCCL
                     reduce-scatter, and the fused peer-store form): key
                     ``splitk_across_gpus``.  At N = 1 the ``families`` key
                     times every other benchmark configuration.
  --impl reference   the reference's CPU path for the same IRs: the torch-CPU
                     statement-level evaluation of the IR (``oracle/interp.py``)
                     over every row of both K2 IRs per step, on every host
                     thread; beside it the torch-CPU family ops and, where a
                     GPU and ``oracle/_ref`` exist, the reference compiler's own
                     PTX for each benchmark configuration timed on the GPU.

One JSON line is printed by rank 0.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
PKG = ROOT / "emmy-ptx-compiler-submission_b200"
for _p in (str(ROOT), str(PKG)):
    if _p not in sys.path:
        sys.path.insert(0, _p)

# Multi-rank runs log NCCL's communicator set-up (ranks, devices, transports)
# to stderr, keeping stdout for the JSON line; set before torch loads NCCL.
if int(os.environ.get("WORLD_SIZE", "1")) > 1:
    if os.environ.get("NCCL_DEBUG", "").upper() not in ("INFO", "TRACE"):
        os.environ["NCCL_DEBUG"] = "INFO"
    os.environ.setdefault("NCCL_DEBUG_SUBSYS", "INIT")
    os.environ.setdefault("NCCL_DEBUG_FILE", "/dev/stderr")

METRIC = "per-family HBM GB/s (K2: softmax4d + layernorm f32)"
UNIT = "GB/s"
K2_WORKLOAD = "K2: softmax f32 [32,16,512,512] dim=-1 + layernorm f32 affine [16384,1024]"
FALLBACK_HBM_GBS = 6650.0
FALLBACK_TENSOR_TFLOPS = 1590.0
# FP32 CUDA-core peak, nominal: 148 SMs x 128 FMA/clk x 2 flops x 1.965 GHz
FP32_NOMINAL_TFLOPS = 148 * 128 * 2 * 1.965e9 / 1e12
# FP64 CUDA-core peak, nominal: 148 SMs x 64 DFMA/clk x 2 flops x 1.965 GHz
FP64_NOMINAL_TFLOPS = 148 * 64 * 2 * 1.965e9 / 1e12
# measured once on this pool's B200s (independent FFMA / DFMA chains on every
# SM at 1965 MHz): 70.86 and 33.35 TFLOP/s
FP32_MEASURED_TFLOPS = 70.86
FP64_MEASURED_TFLOPS = 33.35
# MUFU ex2 rate, nominal: 16 per SM per clock x 148 SMs x 1.965 GHz
MUFU_EXP_PER_S = 16 * 148 * 1.965e9
L2_FLUSH_BYTES = 256 << 20
# Family timings keep each launch's data out of L2: a kernel whose tensors
# total less than this runs on several copies of them, launched back to back
# (the per-launch time is the pass over all copies divided by their number).
FOOTPRINT_BYTES = 256 << 20
MAX_COPIES = 64
# A device spin queued before each timed region keeps the GPU busy while the
# host enqueues the launches, so the CUDA events bracket device work only.  A
# launch through ctypes takes the host several microseconds, longer than a
# small kernel runs, so a timed pass of many launches spins SPIN_PER_LAUNCH
# cycles more per launch (~15 us at 1.965 GHz): every launch is queued before
# the start event fires and the kernels run back to back.
SPIN_CYCLES = 200_000
SPIN_PER_LAUNCH = 30_000

# ncu summary (profiles/) holding each configuration's dram bytes per launch
PROFILE_OF = {
    "K2a_softmax_32x16x512x512": "softmax_f32_K2a.md",
    "K2b_layernorm_16384x1024": "layernorm_f32_K2b.md",
    "K1_rmsnorm_4096x512": "rmsnorm_f32_K1.md",
    "K4b_matvec_f64_16384": "matvec_f64_K4b.md",
    "K4a_splitk_f32_256x65536x256": "gemm_f32_K4a.md",
    "K3a_gemm_f16_4096x2048x8192_bias_relu": "gemm_f16_K3a.md",
    "K3b_bmm_f16_64x512": "bmm_f16_K3b.md",
    "K5_attention_f16_8x32x512x128": "attention_f16_K5.md",
    "K5_sweep_f16_8x32_S512_D256": "attention_f16_D256.md",
    "K5_sweep_f16_8x32_S512_D16": "attention_f16_D16.md",
    "F8a_pointwise_add_f32_2^26": "pointwise_F8.md",
    "F8c_pointwise_bias_relu_f32_16384x4096": "pointwise_broadcast.md",
    "X_softmax_f16_16384x4096": "rowop_softmax_f16.md",
    "F8b_pointwise_gelu_tanh_f16_16384x4096": "pointwise_gelu_f16_F8b.md",
    "F8d_pointwise_int_add_i32_2^26": "pointwise_int_F8d_F8e.md#F8d",
    "F8e_pointwise_int_u8_sub_clamp_2^26": "pointwise_int_F8d_F8e.md#F8e",
}


def _peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return json.loads(p.read_text())
        except ValueError:
            pass
    return {}


def hbm_peak():
    try:
        return float(_peaks()["hbm_gbs"]), "measured"
    except (KeyError, TypeError, ValueError):
        return FALLBACK_HBM_GBS, "fallback"


def tensor_peak():
    try:
        return float(_peaks()["bf16_tflops"]), "measured"
    except (KeyError, TypeError, ValueError):
        return FALLBACK_TENSOR_TFLOPS, "fallback"


def profile_traffic(name):
    """dram bytes per launch recorded from an ncu capture in profiles/<name>
    (``file.md#TAG`` reads the line ``dram_bytes_per_launch (TAG):``)."""
    if not name:
        return None
    name, _, tag = name.partition("#")
    key = f"dram_bytes_per_launch ({tag}):" if tag else "dram_bytes_per_launch:"
    p = ROOT / "profiles" / name
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        if line.strip().startswith(key):
            try:
                return int(line.split(":", 1)[1].strip().split()[0])
            except ValueError:
                return None
    return None


def k2_workload():
    from emmy_ir import synth
    sm = synth.softmax([32, 16, 512, 512], x_init={"dist": "normal", "std": 2.0},
                       entry="k_softmax_K2a")
    ln = synth.layernorm(16384, 1024, eps=1e-5, entry="k_layernorm_K2b",
                         g_init={"dist": "uniform", "low": 0.5, "high": 1.5},
                         b_init={"dist": "normal", "std": 0.1})
    return [sm, ln]


def plan_bytes(plan):
    """Algorithmic bytes of one launch: each tensor argument moved once."""
    from ptxc.launch import torch_dtype
    import torch
    total = 0
    for spec in plan["tensors"].values():
        numel = math.prod(spec["shape"]) if spec["shape"] else 1
        total += numel * torch.empty((), dtype=torch_dtype(spec["dtype"])).element_size()
    return total


def plan_flops(plan):
    if "gemm" in plan:
        g = plan["gemm"]
        return 2.0 * g["batch"] * g["m"] * g["n"] * g["k"]
    if "attention" in plan:
        a = plan["attention"]
        return 2.0 * a["batch"] * a["sq"] * a["sk"] * (a["d"] + a["dv"])
    return 0.0


def shard_inputs(meta, slices, rank, world):
    """Seeded host inputs of this rank's shard: the tensors the shard slices are
    drawn for the slice alone (seeded per rank), the replicated ones whole (the
    same on every rank).  At world = 1 this is ``synth.make_inputs(meta)``."""
    import numpy as np
    from emmy_ir import synth
    if world == 1:
        return synth.make_inputs(meta)
    out = {}
    full = {a["name"]: (math.prod(a["shape"]) if a["shape"] else 1) for a in meta["args"]}
    for a in meta["args"]:
        name = a["name"]
        off, cnt = slices.get(name, (0, full[name]))
        if a.get("output"):
            out[name] = np.zeros(cnt, dtype=synth.NP.get(a["dtype"], np.float32))
        elif cnt == full[name] or "data" in a:
            v = synth.make_inputs(meta, only={name})[name]
            out[name] = v[off:off + cnt] if cnt != full[name] else v
        else:
            shard_meta = {"args": [dict(a, shape=[cnt])]}
            out[name] = synth.make_inputs(shard_meta, seed_offset=1000 * rank)[name]
    return out


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.path = None

    def __enter__(self):
        try:
            fd, self.path = tempfile.mkstemp(suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        if not self.path or not os.path.exists(self.path):
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in Path(self.path).read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for nm, val in zip(names, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(nm)
        os.unlink(self.path)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


class L2Flush:
    """Evict L2 between timed steps: write one 256 MiB buffer, then read another.

    The read pass leaves L2 full of clean lines, so the next timed kernel does
    not pay for writing back the flush's dirty lines.
    """

    def __init__(self, device):
        import torch
        self.w = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device=device)
        self.r = torch.zeros(L2_FLUSH_BYTES // 4, dtype=torch.int32, device=device)

    def __call__(self):
        self.w.zero_()
        self.sink = self.r.sum()


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def cpu_model():
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def cpu_threads():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


# --------------------------------------------------------------------- CPU legs


def cpu_inputs(workload, hosts=None):
    """CPU tensors for the IR evaluation (reusing the bench's host inputs when given)."""
    import torch
    from emmy_ir import synth
    out = []
    for i, (kop, meta) in enumerate(workload):
        if hosts is not None:
            bufs = {k: v for k, v in hosts[i].items()}
        else:
            bufs = {k: torch.from_numpy(v) for k, v in synth.make_inputs(meta).items()}
        for name in [a["name"] for a in meta["args"] if a.get("output")]:
            bufs[name] = torch.zeros_like(bufs[name])
        out.append(bufs)
    return out


def cpu_full_step(workload, bufs_list, threads):
    """One full K2 step of the torch-CPU IR evaluation: every row of both IRs.

    Returns (GB/s over the step's algorithmic bytes, seconds, description).
    """
    import torch
    from oracle.interp import IRInterpreter
    from ptxc import Lowerer
    torch.set_num_threads(threads)
    total_bytes, total_s, desc = 0.0, 0.0, []
    for (kop, meta), bufs in zip(workload, bufs_list):
        plan = Lowerer(kop, meta).plan()
        grid = meta["grid"][0]
        t0 = time.perf_counter()
        with torch.no_grad():
            IRInterpreter(kop, meta, bufs, blocks=(0, grid)).run()
        dt = time.perf_counter() - t0
        total_bytes += plan_bytes(plan)
        total_s += dt
        desc.append(f"{kop.name}: all {grid} rows")
    return total_bytes / total_s / 1e9, total_s, "; ".join(desc)


def cpu_warm(workload, bufs_list, threads):
    """A few rows of each IR, to take first-call costs out of the timed step."""
    import torch
    from oracle.interp import IRInterpreter
    torch.set_num_threads(threads)
    for (kop, meta), bufs in zip(workload, bufs_list):
        with torch.no_grad():
            IRInterpreter(kop, meta, bufs, blocks=(0, 64)).run()


def torch_cpu_family_ops(threads, reps=5):
    """The K2 family ops as torch's own CPU kernels (torch.softmax, layer_norm),
    on the K2 shapes: median of ``reps`` after one warm-up; GB/s over the same
    algorithmic bytes."""
    import torch
    import torch.nn.functional as Fn
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(0)
    x = torch.randn(32, 16, 512, 512, generator=g) * 2.0
    xl = torch.randn(16384, 1024, generator=g)
    gamma = torch.rand(1024, generator=g) + 0.5
    beta = torch.randn(1024, generator=g) * 0.1
    y = torch.empty_like(x)

    def t(fn):
        fn()
        ts = []
        for _ in range(reps):
            t0 = time.perf_counter()
            fn()
            ts.append(time.perf_counter() - t0)
        return statistics.median(ts)
    ts = t(lambda: torch.softmax(x, dim=-1, out=y))
    tl = t(lambda: Fn.layer_norm(xl, (1024,), gamma, beta, 1e-5))
    sm_bytes = 2 * x.numel() * 4
    ln_bytes = 2 * xl.numel() * 4 + 2 * 1024 * 4
    return {"softmax_ms": round(ts * 1e3, 2), "layernorm_ms": round(tl * 1e3, 2),
            "value": round((sm_bytes + ln_bytes) / (ts + tl) / 1e9, 3), "unit": UNIT,
            "threads": threads,
            "ops": "torch.softmax(x, -1) over [32,16,512,512] + F.layer_norm over [16384,1024]"}


# ------------------------------------------------------------------ GPU timing


def _event_pair():
    import torch
    return torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)


def time_launches(make_launch, nbytes, flush, reps=10, warmup=3):
    """Per-launch device time (us) of one kernel configuration.

    ``make_launch()`` returns a zero-argument function that launches the
    kernel on its own copy of the tensors (on the current stream).  With fewer
    than FOOTPRINT_BYTES per launch, ``copies`` such copies run back to back in
    each timed pass, captured once into a CUDA graph and replayed, so the host
    cost of a launch through ctypes (longer than a small kernel) stays out of
    the pass; the time is divided by the number of copies.  Every launch reads
    from HBM, and the 1 us event resolution is spread over many launches.  L2
    is flushed before each timed pass.  Returns (median us per launch, copies).
    """
    import torch
    copies = 1 if nbytes >= FOOTPRINT_BYTES else min(MAX_COPIES,
                                                     -(-FOOTPRINT_BYTES // max(nbytes, 1)))
    fns = [make_launch() for _ in range(copies)]
    for _ in range(warmup):
        for f in fns:
            f()
    torch.cuda.synchronize()
    graph = None
    if copies > 1:
        try:
            side = torch.cuda.Stream()
            side.wait_stream(torch.cuda.current_stream())
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=side):
                for f in fns:
                    f()
            graph.replay()
            torch.cuda.synchronize()
        except RuntimeError:
            graph = None
            torch.cuda.synchronize()
    samples = []
    for _ in range(reps):
        flush()
        torch.cuda._sleep(SPIN_CYCLES + (0 if graph else SPIN_PER_LAUNCH * copies))
        e0, e1 = _event_pair()
        e0.record()
        if graph is not None:
            graph.replay()
        else:
            for f in fns:
                f()
        e1.record()
        e1.synchronize()
        samples.append(e0.elapsed_time(e1) * 1e3 / copies)
    del graph, fns
    return statistics.median(samples), copies


def roofline_block(name, nbytes, flops, us, pipe, n_exp=0, gpus=1):
    """The binding roof of one configuration: t_roof = max(bytes / HBM peak,
    flops / peak of the pipe the kernel uses, exponentials / MUFU rate);
    frac = t_roof / measured time.  The exponential term (attention: one per
    score, B*H*Sq*Sk) uses the nominal MUFU rate, 16 ex2 per SM per clock at
    148 SMs and 1.965 GHz.  With ``gpus`` > 1 the problem is split over that
    many GPUs and every peak is the single-GPU one times ``gpus``."""
    hbm, hsrc = hbm_peak()
    hbm = round(hbm * gpus, 1)
    t_hbm = nbytes / (hbm * 1e9)
    pipe_peak = {"tensor": tensor_peak()[0], "fp32": FP32_MEASURED_TFLOPS,
                 "fp64": FP64_MEASURED_TFLOPS}.get(pipe)
    pipe_peak = round(pipe_peak * gpus, 2) if pipe_peak else None
    t_pipe = flops / (pipe_peak * 1e12) if pipe_peak else 0.0
    t_exp = n_exp / (MUFU_EXP_PER_S * gpus)
    t = us * 1e-6
    if t_hbm >= max(t_pipe, t_exp):
        blk = {"bound": "hbm", "achieved": round(nbytes / t / 1e9, 1), "peak": hbm, "unit": "GB/s",
               "peak_source": f"{hsrc} hbm_gbs"}
    elif t_exp > t_pipe:
        blk = {"bound": "mufu", "achieved": round(n_exp / t / 1e12, 3),
               "peak": round(MUFU_EXP_PER_S / 1e12, 3), "unit": "Texp/s",
               "peak_source": "nominal: 16 ex2 / SM / clock x 148 SMs x 1.965 GHz"}
    else:
        blk = {"bound": pipe, "achieved": round(flops / t / 1e12, 2), "peak": pipe_peak,
               "unit": "TFLOP/s",
               "peak_source": ("measured bf16_tflops (burst)" if pipe == "tensor"
                               else f"measured {pipe} FMA chains")}
    if blk["bound"] == "mufu":
        blk["peak"] = round(MUFU_EXP_PER_S * gpus / 1e12, 3)
    if gpus > 1:
        blk["peak_source"] += f" x {gpus} GPUs"
    blk["frac"] = round(max(t_hbm, t_pipe, t_exp) / t, 4)
    blk["algorithmic_bytes"] = int(nbytes)
    blk["traffic"] = profile_traffic(PROFILE_OF.get(name)) if gpus == 1 else None
    blk["profile"] = PROFILE_OF.get(name) if blk["traffic"] is not None else None
    return blk


def family_cases():
    from emmy_ir import synth
    return {
        "K1_rmsnorm_4096x512": synth.rmsnorm(4096, 512, eps=1e-6),
        "K2a_softmax_32x16x512x512": synth.softmax([32, 16, 512, 512]),
        "K2b_layernorm_16384x1024": synth.layernorm(16384, 1024),
        "K4b_matvec_f64_16384": synth.matvec(16384, 16384),
        "K4a_splitk_f32_256x65536x256": synth.matmul(256, 256, 65536, splits=64, tm=128, tn=128,
                                                     rm=8, rn=8),
        "K3a_gemm_f16_4096x2048x8192_bias_relu": synth.matmul(
            4096, 8192, 2048, dtype="f16", out_dtype="f16", bias=True, relu=True, tm=128, tn=128,
            rm=8, rn=8),
        "K3b_bmm_f16_64x512": synth.matmul(512, 512, 512, batch=64, dtype="f16", out_dtype="f16",
                                           tm=128, tn=128, rm=8, rn=8),
        "K3a_gemm_f16_f32out_4096x2048x8192_bias_relu": synth.matmul(
            4096, 8192, 2048, dtype="f16", out_dtype="f32", bias=True, relu=True, tm=128, tn=128,
            rm=8, rn=8),
        "K3b_bmm_f16_f32out_64x512": synth.matmul(512, 512, 512, batch=64, dtype="f16",
                                                  out_dtype="f32", tm=128, tn=128, rm=8, rn=8),
        "K5_attention_f16_8x32x512x128": synth.attention(8, 32, 512, 128, dtype="f16"),
        **{f"K5_sweep_f16_8x32_S{S}_D{D}": synth.attention(8, 32, S, D, dtype="f16")
           for D in (16, 32, 64, 96, 256) for S in (16, 128, 512)},
        "X_gemm_f64_2048x2048x2048": synth.matmul(2048, 2048, 2048, dtype="f64", tm=128, tn=128,
                                                  rm=8, rn=8, bk=16),
        "X_gemm_f16_8192x8192x8192": synth.matmul(8192, 8192, 8192, dtype="f16", out_dtype="f16",
                                                  tm=128, tn=128, rm=8, rn=8),
        "F8a_pointwise_add_f32_2^26": synth.pointwise(1 << 26, ("add", "x0", "x1"), "f32"),
        "F8b_pointwise_gelu_tanh_f16_16384x4096": synth.pointwise(
            16384 * 4096, ("gelu_tanh", "x0"), "f16", shape=[16384, 4096]),
        "F8c_pointwise_bias_relu_f32_16384x4096": synth.pointwise(
            16384 * 4096, ("relu", ("add", "x0", ("bcast", "b", 4096, 1, 4096))), "f32",
            shape=[16384, 4096]),
        "X_softmax_f16_16384x4096": synth.retype(*synth.softmax([16384, 4096]), "f16", acc="f32"),
        # integer programs (the reference's integer Assign path)
        "F8d_pointwise_int_add_i32_2^26": synth.pointwise(1 << 26, ("add", "x0", "x1"), "i32"),
        "F8e_pointwise_int_u8_sub_clamp_2^26": synth.pointwise(
            1 << 26, ("maximum", ("subtract", "x0", "x1"), ("imm", 0)), "u8"),
    }


def _pipe_of(plan):
    fam = plan["family"]
    if fam == "gemm_f32":
        return "fp32"
    if fam == "gemm_f64":
        return "fp64"
    if fam in ("gemm_f16", "attention_f16"):
        return "tensor"
    return None


def family_extras(device, only=None):
    """Kernel-only time, throughput and roofline of every benchmark configuration."""
    import torch
    from emmy_ir import synth
    from ptxc import Lowerer
    from ptxc.launch import Executor
    out = {}
    flush = L2Flush(device)
    for name, (kop, meta) in family_cases().items():
        if only and not any(o in name for o in only):
            continue
        plan = Lowerer(kop, meta).plan()
        nbytes = plan_bytes(plan)

        def make():
            ex = Executor(plan, device=device)
            for t in ex.tensors.values():
                if t.is_floating_point():
                    t.normal_()
            for a in meta["args"]:
                if "data" in a:
                    ex.tensors[a["name"]].fill_(float(a["data"][0]))
            return ex.launch
        try:
            us, copies = time_launches(make, nbytes, flush)
        except Exception as e:                # a configuration that fails is reported, not fatal
            out[name] = {"error": f"{type(e).__name__}: {e}"[:300]}
            torch.cuda.empty_cache()
            continue
        flops = plan_flops(plan)
        row = {"us": round(us, 2), "gbs": round(nbytes / us / 1e3, 1), "bytes": nbytes,
               "launches_per_sample": copies, "kernel_family": plan["family"]}
        if flops:
            row["tflops"] = round(flops / us / 1e6, 2)
            if plan["family"] == "gemm_f32":
                row["frac_fp32_nominal"] = round(row["tflops"] / FP32_NOMINAL_TFLOPS, 3)
            elif plan["family"] == "gemm_f64":
                row["frac_fp64_nominal"] = round(row["tflops"] / FP64_NOMINAL_TFLOPS, 3)
            elif _pipe_of(plan) == "tensor":
                row["frac_tensor"] = round(row["tflops"] / tensor_peak()[0], 3)
        n_exp = 0
        if "attention" in plan:
            at = plan["attention"]
            n_exp = at["batch"] * at["sq"] * at["sk"]
        row["roofline"] = roofline_block(name, nbytes, flops, us, _pipe_of(plan), n_exp)
        out[name] = row
        torch.cuda.empty_cache()
    if only:
        del flush
        return out
    # the matmul + bias + ReLU package at the K3a size: two kernels (product
    # written as f16, then bias + ReLU) against the fused epilogue launch
    from ptxc.package import Chain, ChainExecutor
    chain = Chain.from_kernels(synth.mm_bias_relu_chain(
        4096, 8192, 2048, dtype="f16", c_dtype="f16", out_dtype="f16", tm=128, tn=128, rm=8, rn=8))
    row = {}
    for fuse in (True, False):
        ex = ChainExecutor(chain, device=device, fuse=fuse)
        for t in ex.buffers.values():
            t.normal_(std=0.02)
        n = ex.launch()
        us, _ = time_launches(lambda: ex.launch, FOOTPRINT_BYTES, flush)
        key = "fused" if fuse else "two_launches"
        row[key + "_us"] = round(us, 2)
        row[key + "_launches"] = n
        row[key + "_tflops"] = round(2.0 * 4096 * 8192 * 2048 / us / 1e6, 2)
        del ex
    out["F2_chain_mm_bias_relu_f16_4096x2048x8192"] = row
    # K1 from a CUDA graph of 16 launches over separate input/output pairs
    kop, meta = synth.rmsnorm(4096, 512, eps=1e-6)
    plan = Lowerer(kop, meta).plan()
    exs = [Executor(plan, device=device) for _ in range(16)]
    for ex in exs:
        for t in ex.tensors.values():
            t.normal_()
        for a in meta["args"]:
            if "data" in a:
                ex.tensors[a["name"]].fill_(float(a["data"][0]))
    side = torch.cuda.Stream(device=device)
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for ex in exs:
            ex.launch()
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        for ex in exs:
            ex.launch()
    us, _ = time_launches(lambda: graph.replay, FOOTPRINT_BYTES, flush)
    us /= len(exs)
    nb = plan_bytes(plan)
    out["K1_rmsnorm_4096x512_graph16"] = {"us_per_launch": round(us, 2),
                                          "gbs": round(nb / us / 1e3, 1),
                                          "launches": len(exs),
                                          "roofline": roofline_block("K1_rmsnorm_4096x512", nb, 0,
                                                                     us, None)}
    del graph, exs
    del flush
    torch.cuda.empty_cache()
    return out


def family_extras_sharded(device, world, rank, max_over_ranks, barrier):
    """Every benchmark configuration split over the ``world`` GPUs of the run.

    Each rank launches its ``ptxc.dist.shard_plan`` shard (rows, batches or
    elements; no collective on the data path) and times it alone as
    ``time_launches`` does at one GPU; the configuration's time is the max over
    ranks, its throughput the whole problem's bytes or flops over that time,
    and its roofline is against ``world`` times the single-GPU peaks.  K4a is
    left out (its K split is the ``splitk_across_gpus`` key) and so is the
    attention shape sweep.  Every rank takes the same collective steps: a
    barrier and one max per configuration, in ``family_cases`` order.
    """
    import torch
    from ptxc import Lowerer
    from ptxc.dist import shard_plan
    from ptxc.launch import Executor
    out = {}
    flush = L2Flush(device)
    for name, (kop, meta) in family_cases().items():
        if name.startswith(("K4a", "K5_sweep")):
            continue
        plan = Lowerer(kop, meta).plan()
        try:
            sub, _ = shard_plan(plan, rank, world)
        except ValueError as e:
            out[name] = {"unsharded": str(e)}
            continue
        nbytes, flops = plan_bytes(plan), plan_flops(plan)

        def make():
            ex = Executor(sub, device=device)
            for t in ex.tensors.values():
                if t.is_floating_point():
                    t.normal_()
            for a in meta["args"]:
                if "data" in a:
                    ex.tensors[a["name"]].fill_(float(a["data"][0]))
            return ex.launch
        barrier()
        # a rank whose configuration fails still takes the same collective
        # steps (its time counts as infinite), so the ranks stay in step
        err = None
        try:
            us, copies = time_launches(make, plan_bytes(sub), flush)
        except Exception as e:
            us, copies, err = float("inf"), 0, f"{type(e).__name__}: {e}"[:300]
        us = max_over_ranks(us)
        if not math.isfinite(us):
            out[name] = {"error": err or "failed on another rank"}
            torch.cuda.empty_cache()
            continue
        row = {"us": round(us, 2), "gbs": round(nbytes / us / 1e3, 1), "bytes": nbytes,
               "launches_per_sample": copies, "kernel_family": plan["family"],
               "gpus": world, "shard_bytes_rank0": plan_bytes(sub)}
        if flops:
            row["tflops"] = round(flops / us / 1e6, 2)
        n_exp = 0
        if "attention" in plan:
            at = plan["attention"]
            n_exp = at["batch"] * at["sq"] * at["sk"]
        row["roofline"] = roofline_block(name, nbytes, flops, us, _pipe_of(plan), n_exp,
                                         gpus=world)
        out[name] = row
        torch.cuda.empty_cache()
    del flush
    return out


def splitk_across_gpus(world, rank, device, reps=10):
    """K4a (256 x 65536 x 256 f32, 64 K partitions) split across the ranks.

    Each rank multiplies its K slice (65536 / N, 64 / N partitions) into a full
    partial C; then (a) the NCCL reduce-scatter leaves each rank its 256 / N
    rows of C, or (b) the fused kernel stores each partial row straight into
    its owner's slot over NVLink and the owner sums its slots, or (c) with no
    host barrier, every rank publishes its step into the others' flag words
    and sums its rows of every partial over NVLink (``splitk_pull_step``).
    Device times, max over ranks, median of ``reps``.  The forms' results are
    compared.
    """
    import ctypes
    import torch
    import torch.distributed as dist
    from ptxc.dist import (PeerPartials, PeerRows, reduce_scatter_rows, shard_ranges,
                           splitk_pull_gemm, splitk_pull_reduce, splitk_to_peers, sum_slots)
    from ptxc.launch import _check, _stream_handle, load_library
    lib = load_library()
    M, N, K = 256, 256, 65536
    k0, k1 = shard_ranges(K, world)[rank]
    kk = k1 - k0
    splits = max(1, 64 // world)
    g = torch.Generator(device=device).manual_seed(4242 + rank)
    A = torch.rand(M, kk, device=device, generator=g) * 2 - 1
    B = torch.rand(kk, N, device=device, generator=g) * 2 - 1
    c_part = torch.empty(M, N, device=device)
    flush = L2Flush(device)
    st = torch.cuda.current_stream()

    def gemm():
        _check(lib.emmy_gemm_f32(ctypes.c_void_p(A.data_ptr()), ctypes.c_void_p(B.data_ptr()),
                                 None, ctypes.c_void_p(c_part.data_ptr()), 1, M, N, kk, 0, 0, 0,
                                 splits, 0, 0, _stream_handle(st)), "emmy_gemm_f32")

    rows = None
    for _ in range(3):
        gemm()
        rows = reduce_scatter_rows(c_part)
    t_g, t_r, t_t = [], [], []
    for _ in range(reps):
        flush()
        torch.cuda.synchronize()
        dist.barrier()
        e0, e1 = _event_pair()
        e2 = torch.cuda.Event(enable_timing=True)
        e0.record()
        gemm()
        e1.record()
        rows = reduce_scatter_rows(c_part)
        e2.record()
        e2.synchronize()
        t_g.append(e0.elapsed_time(e1) * 1e3)
        t_r.append(e1.elapsed_time(e2) * 1e3)
        t_t.append(e0.elapsed_time(e2) * 1e3)
    # fused: GEMM + scatter of partial rows over NVLink, then the slot sum
    slots = torch.zeros(world, M // world, N, device=device)
    peers = PeerRows(slots)
    t_f, t_k, t_s = [], [], []
    try:
        mine = None
        for i in range(3 + reps):
            flush()
            torch.cuda.synchronize()
            dist.barrier()
            e0, e1 = _event_pair()
            e0.record()
            splitk_to_peers(A, B, peers, M, N, splits=splits)
            e1.record()
            torch.cuda.synchronize()
            dist.barrier()
            e2, e3 = _event_pair()
            e2.record()
            mine = sum_slots(peers)
            e3.record()
            e3.synchronize()
            if i >= 3:
                t_k.append(e0.elapsed_time(e1) * 1e3)
                t_s.append(e2.elapsed_time(e3) * 1e3)
                t_f.append(t_k[-1] + t_s[-1])
        diff = float((mine - rows).abs().max()) / max(float(rows.abs().max()), 1e-30)
    finally:
        torch.cuda.synchronize()
        dist.barrier()
        peers.close()
    # pull: GEMM into this step's partial buffer, then the exchange over peer memory
    pp = PeerPartials(M, N, device)
    t_p, t_pg, t_px = [], [], []
    try:
        mine_p = None
        for i in range(3 + reps):
            flush()
            torch.cuda.synchronize()
            dist.barrier()
            e0, e1 = _event_pair()
            em = torch.cuda.Event(enable_timing=True)
            e0.record()
            splitk_pull_gemm(A, B, pp, splits=splits)
            em.record()
            mine_p = splitk_pull_reduce(pp)
            e1.record()
            e1.synchronize()
            if i >= 3:
                t_p.append(e0.elapsed_time(e1) * 1e3)
                t_pg.append(e0.elapsed_time(em) * 1e3)
                t_px.append(em.elapsed_time(e1) * 1e3)
        code = ctypes.c_int(0)
        lib.emmy_get_device_status(ctypes.byref(code), None)
        if code.value:
            raise RuntimeError(f"emmy_peer_reduce_rows: device status {code.value:#x}")
        diff_p = float((mine_p - rows).abs().max()) / max(float(rows.abs().max()), 1e-30)
    finally:
        torch.cuda.synchronize()
        dist.barrier()
        pp.close()
    med = torch.tensor([statistics.median(x) for x in (t_g, t_r, t_t, t_k, t_s, t_f)] +
                       [max(diff, diff_p), statistics.median(t_p), statistics.median(t_pg),
                        statistics.median(t_px)],
                       device=device, dtype=torch.float64)
    dist.all_reduce(med, op=dist.ReduceOp.MAX)
    v = [float(x) for x in med.tolist()]
    flops = 2.0 * M * N * K
    del flush
    return {"config": f"{M}x{K}x{N} f32, K split over {world} GPUs ({splits} partitions per GPU)",
            "gemm_us": round(v[0], 2), "reduce_scatter_us": round(v[1], 2),
            "total_us": round(v[2], 2), "total_tflops": round(flops / v[2] / 1e6, 2),
            "fused_kernel_us": round(v[3], 2), "fused_slot_sum_us": round(v[4], 2),
            "fused_total_us": round(v[5], 2), "fused_tflops": round(flops / v[5] / 1e6, 2),
            "pull_gemm_us": round(v[8], 2), "pull_exchange_us": round(v[9], 2),
            "pull_total_us": round(v[7], 2), "pull_tflops": round(flops / v[7] / 1e6, 2),
            "forms_agree_max_rel": v[6],
            "timing": "device events per rank, max over ranks, median of 10; L2 flushed"}


# ------------------------------------------------------------------- the arms


def run_reference_arm(args):
    from ptxc import Lowerer
    world, rank, _ = dist_setup()
    if rank != 0:
        return 0
    threads = cpu_threads()
    workload = k2_workload()
    bufs = cpu_inputs(workload)
    cpu_warm(workload, bufs, threads)
    # one whole step untimed (first touch of the outputs), then the timed
    # steps, capped so the arm ends within a few minutes on a slow host (the
    # line reports the number actually timed)
    _, first_s, desc = cpu_full_step(workload, bufs, threads)
    steps = args.steps
    budget_s = float(os.environ.get("EMMY_REFERENCE_BUDGET_S", "240"))
    if first_s * steps > budget_s:
        steps = max(1, int(budget_s // max(first_s, 1e-9)))
    per_step = []
    for _ in range(steps):
        _, secs, desc = cpu_full_step(workload, bufs, threads)
        per_step.append(secs)
    total_s = sum(per_step)
    step_bytes = sum(plan_bytes(Lowerer(k, m).plan()) for k, m in workload)
    value = steps * step_bytes / total_s / 1e9
    line = {
        "metric": METRIC, "value": round(value, 4), "unit": UNIT, "n_gpus": args.gpus,
        "steps": steps, "steps_requested": args.steps, "warmup": 1,
        "ms_per_step": round(1000 * total_s / steps, 3),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded numpy inputs, BASELINE distributions)", "impl": "reference",
        "config": {"workload": K2_WORKLOAD,
                   "reference_path": "torch-CPU statement-level evaluation of the same IR "
                                     "(oracle/interp.py) over every row of both IRs per step",
                   "bytes_per_step": step_bytes},
        "cpu_baseline": {"value": round(value, 4), "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": desc + " (the whole K2 step, every step)",
                         "cpu_model": cpu_model()},
        "e2e": {"value": round(value, 4), "unit": UNIT, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "torch_cpu_family_ops": torch_cpu_family_ops(threads),
    }
    if not args.no_families:
        line["reference_ptx"] = reference_ptx_families()
    print(json.dumps(line), flush=True)
    return 0


def reference_ptx_families():
    """The reference compiler's own PTX (oracle/_ref, made by the unmodified
    reference compiler) for each benchmark configuration, launched as the
    reference harness launches it, timed on the GPU with the families' protocol."""
    try:
        import torch
        if not torch.cuda.is_available():
            return {"unavailable": "no GPU"}
        from emmy_ir import synth
        from oracle import ref_ptx
        from oracle.make_ref_ptx import BENCH_CASES
        from ptxc import Lowerer
    except ImportError as e:
        return {"unavailable": f"import failed: {e}"}
    names = {"K1_rmsnorm": "K1_rmsnorm_4096x512", "K2a_softmax": "K2a_softmax_32x16x512x512",
             "K2b_layernorm": "K2b_layernorm_16384x1024", "K4b_matvec_f64": "K4b_matvec_f64_16384",
             "K4a_splitk_f32": "K4a_splitk_f32_256x65536x256",
             "K3a_gemm_f16": "K3a_gemm_f16_4096x2048x8192_bias_relu",
             "K3b_bmm_f16": "K3b_bmm_f16_64x512", "K5_attention_f16": "K5_attention_f16_8x32x512x128",
             "F8a_pointwise_add": "F8a_pointwise_add_f32_2^26",
             "F8d_pointwise_int": "F8d_pointwise_int_add_i32_2^26"}
    torch.cuda.set_device(0)
    dev = torch.device("cuda", 0)
    flush = L2Flush(dev)
    from ptxc.launch import torch_dtype
    out = {}
    for name, make in BENCH_CASES.items():
        if not ref_ptx.available(name):
            continue
        kop, meta = make(synth)
        k = ref_ptx.RefKernel(name)
        nbytes = sum((math.prod(a["shape"]) if a["shape"] else 1) *
                     torch.empty((), dtype=torch_dtype(a["dtype"])).element_size()
                     for a in meta["args"])
        # the harness zeroes these before every launch (atomic split-K outputs)
        zero = k.k.get("zero_outputs") or []

        def make_launch():
            ts = {}
            for a in meta["args"]:
                n = math.prod(a["shape"]) if a["shape"] else 1
                t = torch.empty(n, dtype=torch_dtype(a["dtype"]), device=dev)
                if "data" in a:
                    t.fill_(a["data"][0])
                elif a.get("output") or not t.is_floating_point():
                    t.zero_()
                else:
                    t.normal_()
                ts[a["name"]] = t
            zs = [ts[z] for z in zero if z in ts]

            def launch():
                for z in zs:
                    z.zero_()
                k.launch(ts)
            return launch
        us, copies = time_launches(make_launch, nbytes, flush)
        k.close()
        row = {"us": round(us, 2), "gbs": round(nbytes / us / 1e3, 1),
               "launches_per_sample": copies}
        flops = plan_flops(Lowerer(kop, meta).plan())
        if flops:
            row["tflops"] = round(flops / us / 1e6, 2)
        out[names.get(name, name)] = row
        torch.cuda.empty_cache()
    del flush
    return out


def run_b200_arm(args):
    import torch
    import torch.distributed as dist
    from ptxc import Lowerer
    from ptxc.dist import shard_plan
    from ptxc.launch import Executor, load_library

    world, rank, local = dist_setup()
    if world > 1:
        from datetime import timedelta
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=180),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(0)
    device = torch.device("cuda", torch.cuda.current_device())
    load_library()
    peak, peak_src = hbm_peak()

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], device=device, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    workload = k2_workload()
    full_plans = [Lowerer(k, m).plan() for k, m in workload]
    total_bytes = sum(plan_bytes(p) for p in full_plans)
    # this rank's rows of each IR (the whole plan at N = 1)
    shards = [shard_plan(p, rank, world) for p in full_plans]
    plans = [s for s, _ in shards]
    my_bytes = sum(plan_bytes(p) for p in plans)
    hosts = []
    for (kop, meta), (_, slices) in zip(workload, shards):
        h = shard_inputs(meta, slices, rank, world)
        hosts.append({k: torch.from_numpy(v).pin_memory() for k, v in h.items()})
    execs = [Executor(p, device=device) for p in plans]
    for ex, h in zip(execs, hosts):
        ex.upload(h)
    torch.cuda.synchronize()
    flush = L2Flush(device)

    side = torch.cuda.Stream(device=device)

    def timed_steps(exs, steps):
        """(total ms, softmax-launch ms per step, launches) over ``steps`` steps.

        The two IRs of a step are independent: the layernorm runs on a second
        stream beside the softmax (forked after the start event, joined before
        the end event), so its short launch overlaps the long one.
        """
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True),
               torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
        main = torch.cuda.current_stream()
        launches = 0
        for i in range(steps):
            flush()                         # L2 flush between steps (outside the events)
            torch.cuda._sleep(SPIN_CYCLES)
            e0, e1, e2 = ev[i]
            e0.record(main)
            side.wait_event(e0)
            with torch.cuda.stream(side):
                launches += exs[1].launch(stream=side)   # layernorm
            launches += exs[0].launch(stream=main)       # softmax (dominant kernel)
            e1.record(main)
            main.wait_stream(side)
            e2.record(main)
        torch.cuda.synchronize()
        total = sum(a.elapsed_time(c) for a, b, c in ev)
        return total, [a.elapsed_time(b) for a, b, c in ev], launches

    # ---- device-resident timing: this rank's partition (the headline)
    for _ in range(args.warmup):
        for ex in execs:
            ex.launch()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    clocks = ClockSampler(device.index).__enter__()
    total_ms, sm_ms, launches = timed_steps(execs, args.steps)
    barrier()
    torch.cuda.synchronize()
    total_ms = max_over_ranks(total_ms)
    value = args.steps * total_bytes / (total_ms * 1e-3) / 1e9
    sm_bytes = plan_bytes(plans[0])
    sm_avg = statistics.mean(sm_ms)
    achieved = sm_bytes / (sm_avg * 1e-3) / 1e9

    # ---- end to end through the public API: pinned host -> device -> kernels -> host
    outs = [{name: torch.empty(ex.tensors[name].numel(), dtype=ex.tensors[name].dtype).pin_memory()
             for name in p["outputs"]} for ex, p in zip(execs, plans)]
    h2d = sum(h[n].numel() * h[n].element_size() for ex, h in zip(execs, hosts) for n in ex.inputs())
    d2h = sum(t.numel() * t.element_size() for o in outs for t in o.values())

    def e2e_step():
        # each plan in chunks: H2D, kernels and D2H on three streams, overlapped
        for j, (ex, h, o) in enumerate(zip(execs, hosts, outs)):
            ex.run_pipelined(h, o, join=(j == len(execs) - 1))

    for _ in range(max(2, args.warmup)):
        e2e_step()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    e2e_ev = [_event_pair() for _ in range(args.steps)]
    for i in range(args.steps):
        a, b = e2e_ev[i]
        a.record()
        e2e_step()
        b.record()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(sum(a.elapsed_time(b) for a, b in e2e_ev))
    e2e_value = args.steps * total_bytes / (e2e_ms * 1e-3) / 1e9
    # the e2e roof: this step's own pinned buffers copied both ways at once (the
    # largest input up, the largest output down), best of three, max over ranks
    big_in = max(((ex, h, n) for ex, h in zip(execs, hosts) for n in ex.inputs()),
                 key=lambda t: t[1][t[2]].numel() * t[1][t[2]].element_size())
    big_out = max(((ex, o, n) for ex, o in zip(execs, outs) for n in o),
                  key=lambda t: t[1][t[2]].numel() * t[1][t[2]].element_size())
    pcie_bytes = (big_in[1][big_in[2]].numel() * big_in[1][big_in[2]].element_size() +
                  big_out[1][big_out[2]].numel() * big_out[1][big_out[2]].element_size())
    s_up, s_down = torch.cuda.Stream(device=device), torch.cuda.Stream(device=device)
    best = None
    for _ in range(3):
        torch.cuda.synchronize()
        a, b = _event_pair()
        cur = torch.cuda.current_stream(device)
        a.record(cur)
        s_up.wait_stream(cur)
        s_down.wait_stream(cur)
        with torch.cuda.stream(s_up):
            big_in[0].tensors[big_in[2]].copy_(big_in[1][big_in[2]], non_blocking=True)
        with torch.cuda.stream(s_down):
            big_out[1][big_out[2]].copy_(big_out[0].tensors[big_out[2]], non_blocking=True)
        cur.wait_stream(s_up)
        cur.wait_stream(s_down)
        b.record(cur)
        torch.cuda.synchronize()
        ms = a.elapsed_time(b)
        best = ms if best is None else min(best, ms)
    pcie_gbs = pcie_bytes / (max_over_ranks(best) * 1e-3) / 1e9
    e2e_pcie = (h2d + d2h) * args.steps / (e2e_ms * 1e-3) / 1e9
    # spot check the e2e outputs against the device results of the same step
    for ex, o in zip(execs, outs):
        for name, t in o.items():
            assert torch.equal(t, ex.tensors[name].cpu()), "e2e output mismatch"
    # bytes per step over all ranks (each rank copies its own shard)
    h2d_all = int(round(max_over_ranks(h2d) * world)) if world > 1 else h2d
    d2h_all = int(round(max_over_ranks(d2h) * world)) if world > 1 else d2h
    execs.clear()

    # ---- weak scaling key (N > 1): every rank on a full K2 batch
    weak = None
    if world > 1:
        wexecs = []
        for (kop, meta), p in zip(workload, full_plans):
            ex = Executor(p, device=device)
            for t in ex.tensors.values():
                t.normal_()
            for a in meta["args"]:
                if "data" in a:
                    ex.tensors[a["name"]].fill_(float(a["data"][0]))
            wexecs.append(ex)
        for _ in range(args.warmup):
            for ex in wexecs:
                ex.launch()
        torch.cuda.synchronize()
        barrier()
        wms, _, _ = timed_steps(wexecs, args.steps)
        barrier()
        wms = max_over_ranks(wms)
        weak = {"value": round(world * args.steps * total_bytes / (wms * 1e-3) / 1e9, 2),
                "unit": UNIT, "ms_per_step": round(wms / args.steps, 4),
                "per_rank": "each rank runs one full K2 batch per step"}
        wexecs.clear()
    clocks.__exit__(None, None, None)
    del flush
    torch.cuda.empty_cache()

    splitk = splitk_across_gpus(world, rank, device) if world > 1 else None
    extras = None
    if not args.no_families:
        extras = (family_extras(device) if world == 1 else
                  family_extras_sharded(device, world, rank, max_over_ranks, barrier))

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        # the same measurement as the reference arm: one whole K2 step of the
        # torch-CPU IR evaluation (every row), after a warm-up on a few rows
        threads = cpu_threads()
        bufs = cpu_inputs(workload, hosts)
        cpu_warm(workload, bufs, threads)
        gbs, secs, desc = cpu_full_step(workload, bufs, threads)
        cpu = {"value": round(gbs, 4), "unit": UNIT, "cores": threads, "kind": "port",
               "sample": desc + f" (one whole K2 step, {secs:.1f} s)", "cpu_model": cpu_model()}

    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return 0
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(total_ms / args.steps, 4),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded numpy inputs, BASELINE distributions)",
        "config": {
            "workload": K2_WORKLOAD,
            "parallelism": f"rows partitioned over {world} GPU(s) (ptxc.dist.shard_plan), "
                           "no collective on the data path",
            "bytes_per_step": total_bytes,
            "bytes_per_step_rank0": my_bytes,
            "l2": "flushed between steps (256 MiB device write + read outside the timed events)",
            "ir": "synthesised Kernel IR in the reference fixtures' reduction shapes",
        },
        "roofline": {"bound": "hbm", "kernel": "emmy softmax (row_resident_kernel)",
                     "achieved": round(achieved, 1), "peak": peak, "unit": UNIT,
                     "frac": round(achieved / peak, 4),
                     "peak_source": (f"{peak_src} (MEASURED_PEAKS.json hbm_gbs)"
                                     if peak_src == "measured" else "fallback 6.65 TB/s"),
                     "bytes_per_launch": sm_bytes, "avg_launch_us": round(sm_avg * 1000, 2),
                     "traffic": (profile_traffic("softmax_f32_K2a.md") if world == 1 else None)},
        "e2e": {"value": round(e2e_value, 3), "unit": UNIT, "h2d_bytes_per_step": h2d_all,
                "d2h_bytes_per_step": d2h_all,
                "path": ("ptxc.launch.Executor.run_pipelined: pinned host inputs -> H2D / C-ABI "
                         "kernels / D2H overlapped per ~32 MiB chunk on three streams -> pinned "
                         "host outputs"),
                "roofline": {"bound": "pcie", "achieved": round(e2e_pcie, 2),
                             "peak": round(pcie_gbs, 2), "unit": "GB/s",
                             "frac": round(e2e_pcie / pcie_gbs, 4),
                             "peak_source": ("measured live: the step's largest input up and "
                                             "largest output down at once (pinned), per rank")}},
        "gpu_launches": launches,
        "clocks": clocks.summary(),
    }
    if weak:
        line["weak"] = weak
    if splitk:
        line["splitk_across_gpus"] = splitk
    if cpu:
        line["cpu_baseline"] = cpu
    if extras:
        line["families"] = extras
    print(json.dumps(line), flush=True)
    return 0


PROFILE_CASES = {
    # name: builder -- small cases (inputs above L2, a few hundred MB at most)
    # for one-kernel ncu captures: `python bench.py --case softmax_65536x512`
    "softmax_65536x512": lambda s: s.softmax([65536, 512], x_init={"dist": "normal", "std": 2.0}),
    "softmax_K2a": lambda s: s.softmax([32, 16, 512, 512], x_init={"dist": "normal", "std": 2.0}),
    "layernorm_16384x1024": lambda s: s.layernorm(16384, 1024),
    "rmsnorm_65536x512": lambda s: s.rmsnorm(65536, 512, eps=1e-6),
    "matvec_f64_8192x4096": lambda s: s.matvec(8192, 4096),
    "matvec_f64_K4b": lambda s: s.matvec(16384, 16384),
    "gemm_f16_K3a": lambda s: s.matmul(4096, 8192, 2048, dtype="f16", out_dtype="f16", bias=True,
                                       relu=True, tm=128, tn=128, rm=8, rn=8),
    "gemm_f16_2048": lambda s: s.matmul(2048, 2048, 2048, dtype="f16", out_dtype="f16",
                                        tm=128, tn=128, rm=8, rn=8),
    "attention_f16_K5": lambda s: s.attention(8, 32, 512, 128, dtype="f16"),
    "attention_f16_D256": lambda s: s.attention(8, 32, 512, 256, dtype="f16"),
    "attention_f16_D16": lambda s: s.attention(8, 32, 512, 16, dtype="f16"),
    "attention_f16_D32": lambda s: s.attention(8, 32, 512, 32, dtype="f16"),
    "attention_f16_D96": lambda s: s.attention(8, 32, 512, 96, dtype="f16"),
    "gemm_f32_splitk_K4a": lambda s: s.matmul(256, 256, 65536, splits=64, tm=128, tn=128, rm=8,
                                              rn=8),
    "pointwise_add_2^26": lambda s: s.pointwise(1 << 26, ("add", "x0", "x1"), "f32"),
    "bmm_f16_K3b": lambda s: s.matmul(512, 512, 512, batch=64, dtype="f16", out_dtype="f16",
                                      tm=128, tn=128, rm=8, rn=8),
    "rmsnorm_K1": lambda s: s.rmsnorm(4096, 512, eps=1e-6),
    "pointwise_gelu_f16_2^26": lambda s: s.pointwise(1 << 26, ("gelu_tanh", "x0"), "f16"),
    "pointwise_bias_relu_f32_16384x4096": lambda s: s.pointwise(
        16384 * 4096, ("relu", ("add", "x0", ("bcast", "b", 4096, 1, 4096))), "f32",
        shape=[16384, 4096]),
    "gemm_f64_2048": lambda s: s.matmul(2048, 2048, 2048, dtype="f64", tm=128, tn=128, rm=8, rn=8,
                                        bk=16),
    "rowop_softmax_f16_16384x4096": lambda s: s.retype(*s.softmax([16384, 4096]), "f16", acc="f32"),
    "rowop_layernorm_f16_16384x1024": lambda s: s.retype(*s.layernorm(16384, 1024), "f16",
                                                         acc="f32"),
    "pointwise_int_add_i32_2^26": lambda s: s.pointwise(1 << 26, ("add", "x0", "x1"), "i32"),
    "pointwise_int_u8_sub_clamp_2^26": lambda s: s.pointwise(
        1 << 26, ("maximum", ("subtract", "x0", "x1"), ("imm", 0)), "u8"),
    "gemm_f16_4096_wide_tiles": lambda s: s.matmul(4096, 4096, 4096, dtype="f16", out_dtype="f16",
                                                   tm=128, tn=128, rm=8, rn=8),
}


def run_case(name, launches):
    """Launch one family case a few times (no timing): the target of an ncu capture."""
    import torch
    from emmy_ir import synth
    from ptxc import Lowerer
    from ptxc.launch import Executor
    kop, meta = PROFILE_CASES[name](synth)
    plan = Lowerer(kop, meta).plan()
    ex = Executor(plan, device="cuda:0")
    ex.upload(synth.make_inputs(meta))
    for _ in range(launches):
        ex.launch()
    torch.cuda.synchronize()
    print(json.dumps({"case": name, "family": plan["family"], "launches": launches,
                      "bytes_per_launch": plan_bytes(plan)}))
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--case", choices=sorted(PROFILE_CASES), help="run one profiling case and exit")
    ap.add_argument("--launches", type=int, default=3)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-families", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--families-only", nargs="*", default=None,
                    help="time only the family configurations whose name contains one of these")
    args = ap.parse_args()
    if args.case:
        return run_case(args.case, args.launches)
    if args.families_only is not None:
        import torch
        torch.cuda.set_device(0)
        print(json.dumps(family_extras(torch.device("cuda", 0), only=args.families_only or None)))
        return 0
    if args.warmup < 3 and args.impl == "b200":
        args.warmup = 3
    if args.impl == "reference":
        return run_reference_arm(args)
    return run_b200_arm(args)


if __name__ == "__main__":
    sys.exit(main())
