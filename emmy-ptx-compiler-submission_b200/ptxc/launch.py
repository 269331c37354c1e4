"""Execute a launch plan through ``libemmyb200.so`` (ctypes C-ABI).

This replaces what the reference's harness does with the PTX it emits
(``tools/localrun.py:102-142``: load the module, allocate, copy, launch under
the meta geometry, copy back): here the plan names a C-ABI symbol of the
prebuilt sm_100a library and its tensor roles, and the library picks its own
launch geometry.  Device memory and streams come from PyTorch; the library
itself allocates nothing.

There is no fallback: if the library is missing or a call fails, this raises.
"""

from __future__ import annotations

import ctypes
import math
import os
from pathlib import Path

_HERE = Path(__file__).resolve().parent
DEFAULT_LIB = _HERE.parent / "libemmyb200.so"

_i64 = ctypes.c_int64
_vp = ctypes.c_void_p
_int = ctypes.c_int
_sz = ctypes.c_size_t

# symbol -> argtypes (all return int status)
SIGNATURES = {
    "emmy_version": [],
    "emmy_get_device_status": [ctypes.POINTER(_int), _vp],
    "emmy_zero": [_vp, _sz, _vp],
    "emmy_reduce_f32": [_vp, _vp, _i64, _i64, _i64, _int, _int, _vp, _vp, _sz, _vp],
    "emmy_reduce_workspace_bytes": [_i64, _i64, _i64],
    "emmy_reduce_f32_noalloc": [_vp, _vp, _i64, _int, _int, _vp, _vp],
    "emmy_rownorm_f32": [_vp, _vp, _vp, _vp, _i64, _i64, _vp, _vp, _int, _vp],
    "emmy_softmax_f32": [_vp, _vp, _i64, _i64, _i64, _vp],
    "emmy_matvec_f64": [_vp, _vp, _vp, _i64, _i64, _vp],
    "emmy_rowop": [_vp, _int, _vp, _vp, _int, _vp, _int, _i64, _i64, _i64, _int, _int, _vp, _vp,
                   _int, _int, _vp],
    "emmy_gemm_f32": [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _int, _int, _int, _vp],
    "emmy_gemm_f64": [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _int, _int, _int, _vp],
    "emmy_gemm_f32_rows_to_peers": [_vp, _vp, _vp, _vp, _i64, _int, _int, _i64, _i64, _i64, _i64,
                                    _int, _vp, _vp, _i64, _vp],
    "emmy_ipc_export": [_vp, _vp, _vp],
    "emmy_ipc_import": [_vp, _i64, _vp, _vp],
    "emmy_ipc_close": [_vp],
    "emmy_peer_reduce_rows": [_vp, _vp, _int, _int, _i64, _i64, _i64, _i64, _vp, _vp],
    "emmy_gemm_f16": [_vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _int, _int, _int, _vp],
    "emmy_attention_f32": [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _int, _vp],
    "emmy_attention_f16": [_vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _i64, _int, _int, _vp],
    "emmy_pointwise": [_vp, _vp, _int, _vp, _vp, _int, _vp, _int, _vp, _int, _int, _int, _vp, _int,
                       _i64, _vp],
    "emmy_pointwise_indexed": [_vp, _vp, _vp, _int, _vp, _vp, _int, _vp, _int, _vp, _int, _int, _int,
                               _vp, _int, _i64, _i64, _vp],
    "emmy_pointwise_int": [_vp, _vp, _vp, _int, _vp, _vp, _int, _vp, _int, _vp, _int, _int, _vp,
                           _int, _i64, _i64, _int, _vp],
}
RESTYPES = {"emmy_reduce_workspace_bytes": _sz}

REDUCE_OP = {"sum": 0, "max": 1, "min": 2}
REDUCE_PRE = {"identity": 0, "square": 1, "abs": 2}
NORM_MODE = {"rms": 0, "l2": 1, "layer": 2}
DT_CODE = {"f32": 0, "f16": 1, "f64": 2, "i8": 3, "u8": 4, "i16": 5, "u16": 6, "i32": 7,
           "u32": 8, "i64": 9, "u64": 10}


class LibraryError(RuntimeError):
    pass


_LIB = None


def library_path() -> Path:
    return Path(os.environ.get("EMMY_B200_LIB", str(DEFAULT_LIB)))


def load_library():
    """Load ``libemmyb200.so`` once; raise ``LibraryError`` when it is absent."""
    global _LIB
    if _LIB is not None:
        return _LIB
    path = library_path()
    if not path.exists():
        raise LibraryError(
            f"{path} is missing: build it with `python emmy-ptx-compiler-submission_b200/build.py` "
            "(there is no CPU fallback)")
    lib = ctypes.CDLL(str(path))
    for name, argtypes in SIGNATURES.items():
        fn = getattr(lib, name, None)
        if fn is None:
            continue
        fn.argtypes = argtypes
        fn.restype = RESTYPES.get(name, _int)
    lib.emmy_last_error.argtypes = []
    lib.emmy_last_error.restype = ctypes.c_char_p
    _LIB = lib
    return lib


def _check(rc: int, what: str) -> None:
    if rc != 0:
        msg = load_library().emmy_last_error()
        raise RuntimeError(f"{what} failed (status {rc}): {msg.decode() if msg else ''}")


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream_handle(stream):
    if stream is None:
        import torch
        return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    return ctypes.c_void_p(getattr(stream, "cuda_stream", stream))


_TORCH_DT = None


def torch_dtype(dt: str):
    import torch
    global _TORCH_DT
    if _TORCH_DT is None:
        _TORCH_DT = {"f32": torch.float32, "f16": torch.float16, "f64": torch.float64,
                     "i32": torch.int32, "i64": torch.int64, "i8": torch.int8,
                     "u8": torch.uint8, "bool": torch.bool, "i16": torch.int16,
                     "u16": torch.uint16, "u32": torch.uint32, "u64": torch.uint64}
    return _TORCH_DT[dt]


def check_tensors(plan: dict, tensors: dict) -> None:
    """Every plan tensor present, on a CUDA device, contiguous, right dtype and size."""
    for name, spec in plan["tensors"].items():
        t = tensors.get(name)
        if t is None:
            raise ValueError(f"missing tensor {name!r}")
        if not t.is_cuda:
            raise ValueError(f"tensor {name!r} is not on a CUDA device")
        if not t.is_contiguous():
            raise ValueError(f"tensor {name!r} is not contiguous")
        if t.dtype != torch_dtype(spec["dtype"]):
            raise ValueError(f"tensor {name!r} has dtype {t.dtype}, plan says {spec['dtype']}")
        numel = math.prod(spec["shape"]) if spec["shape"] else 1
        if t.numel() != numel:
            raise ValueError(f"tensor {name!r} has {t.numel()} elements, plan says {numel}")


def workspace_bytes(plan: dict) -> int:
    """Device scratch a plan wants (the caller allocates it)."""
    if plan["family"] == "reduce":
        v = plan["view"]
        return int(load_library().emmy_reduce_workspace_bytes(v["outer"], v["n"], v["inner"]))
    return 0


def run(plan: dict, tensors: dict, stream=None, workspace=None, check: bool = True) -> int:
    """Launch the plan's kernel(s) on ``stream``; returns the number of library launches."""
    lib = load_library()
    if check:
        check_tensors(plan, tensors)
    st = _stream_handle(stream)
    launches = 0
    for name in plan.get("zero_outputs", []):
        t = tensors[name]
        _check(lib.emmy_zero(_ptr(t), t.numel() * t.element_size(), st), "emmy_zero")
        launches += 1
    a = plan["args"]
    p = plan.get("params", {})
    fam = plan["family"]
    T = lambda role: tensors[a[role]] if role in a else None  # noqa: E731
    if fam == "reduce":
        v = plan["view"]
        ws = workspace
        _check(lib.emmy_reduce_f32(_ptr(T("x")), _ptr(T("y")), v["outer"], v["n"], v["inner"],
                                   REDUCE_OP[p["op"]], REDUCE_PRE[p["pre"]], _ptr(T("count")),
                                   _ptr(ws), 0 if ws is None else ws.numel() * ws.element_size(),
                                   st), "emmy_reduce_f32")
        launches += 2 if ws is not None and workspace_bytes(plan) else 1
    elif fam == "rownorm":
        v = plan["view"]
        _check(lib.emmy_rownorm_f32(_ptr(T("x")), _ptr(T("w")), _ptr(T("b")), _ptr(T("y")),
                                    v["outer"], v["n"], _ptr(T("eps")), _ptr(T("count")),
                                    NORM_MODE[p["mode"]], st), "emmy_rownorm_f32")
        launches += 1
    elif fam == "softmax":
        v = plan["view"]
        _check(lib.emmy_softmax_f32(_ptr(T("x")), _ptr(T("y")), v["outer"], v["n"], v["inner"], st),
               "emmy_softmax_f32")
        launches += 1
    elif fam == "rowop":
        v, pr, dt = plan["view"], plan["params"], plan["tensors"]
        mode = {"sum": 0, "max": 1, "min": 2, "softmax": 3, "rms": 4, "l2": 5, "layer": 6,
                "dot": 7}[pr["mode"]]
        _check(lib.emmy_rowop(_ptr(T("x")), DT_CODE[dt[a["x"]]["dtype"]], _ptr(T("w")), _ptr(T("b")),
                              DT_CODE[pr["wb_dtype"]], _ptr(T("y")), DT_CODE[dt[a["y"]]["dtype"]],
                              v["outer"], v["n"], v["inner"], mode, REDUCE_PRE[pr["pre"]],
                              _ptr(T("eps")), _ptr(T("count")), DT_CODE[pr["const_dtype"]],
                              int(pr["compute"] == "f64"), st), "emmy_rowop")
        launches += 1
    elif fam == "matvec":
        v = plan["view"]
        _check(lib.emmy_matvec_f64(_ptr(T("x")), _ptr(T("v")), _ptr(T("y")), v["outer"], v["n"], st),
               "emmy_matvec_f64")
        launches += 1
    elif fam in ("gemm_f32", "gemm_f64"):
        g = plan["gemm"]
        fn = lib.emmy_gemm_f32 if fam == "gemm_f32" else lib.emmy_gemm_f64
        _check(fn(_ptr(T("a")), _ptr(T("b")), _ptr(T("bias")), _ptr(T("c")),
                  g["batch"], g["m"], g["n"], g["k"], g["a_batch_stride"],
                  g["b_batch_stride"], g["c_batch_stride"], g["splits"],
                  int(g["accumulate"]), g["epilogue"], st), "emmy_" + fam)
        launches += 1
    elif fam == "gemm_f16":
        g = plan["gemm"]
        _check(lib.emmy_gemm_f16(_ptr(T("a")), _ptr(T("b")), _ptr(T("bias")), _ptr(T("c")),
                                 g["batch"], g["m"], g["n"], g["k"], g["out_dtype"],
                                 g["epilogue"], int(g["accumulate"]), st), "emmy_gemm_f16")
        launches += 1
    elif fam == "attention_f32":
        g = plan["attention"]
        _check(lib.emmy_attention_f32(_ptr(T("q")), _ptr(T("k")), _ptr(T("v")), _ptr(T("o")),
                                      _ptr(T("scale")), g["batch"], g["sq"], g["sk"], g["d"],
                                      g["dv"], int(g["k_transposed"]), st), "emmy_attention_f32")
        launches += 1
    elif fam == "attention_f16":
        g = plan["attention"]
        _check(lib.emmy_attention_f16(_ptr(T("q")), _ptr(T("k")), _ptr(T("v")), _ptr(T("o")),
                                      _ptr(T("scale")), g["batch"], g["sq"], g["sk"], g["d"],
                                      g["out_dtype"], int(g["k_transposed"]), st),
               "emmy_attention_f16")
        launches += 1
    elif fam == "pointwise":
        g = plan["pointwise"]
        ins, scs, imms = g["inputs"], g["scalars"], g["immediates"]
        in_ptrs = (_vp * max(1, len(ins)))(*[_ptr(tensors[n]) for n in ins])
        in_dts = (_int * max(1, len(ins)))(*[DT_CODE[plan["tensors"][n]["dtype"]] for n in ins])
        sc_ptrs = (_vp * max(1, len(scs)))(*[_ptr(tensors[n]) for n in scs])
        sc_dts = (_int * max(1, len(scs)))(*[DT_CODE[plan["tensors"][n]["dtype"]] for n in scs])
        imm = (ctypes.c_double * max(1, len(imms)))(*[float(v) for v in imms])
        flat = [int(x) for row in g["program"] for x in row]
        prog = (_int * len(flat))(*flat)
        if "input_index" in g:
            idx = []
            for n, (d, m) in zip(ins, g["input_index"]):
                idx += [int(d), int(m), tensors[n].numel()]
            idx_arr = (ctypes.c_int64 * len(idx))(*idx)
            _check(lib.emmy_pointwise_indexed(in_ptrs, in_dts, idx_arr, len(ins), sc_ptrs, sc_dts,
                                              len(scs), imm, len(imms), prog, len(g["program"]),
                                              g["result_reg"], int(g["compute"] == "f64"),
                                              _ptr(T("out")), DT_CODE[g["out_dtype"]],
                                              int(g.get("first", 0)), g["n"], st),
                   "emmy_pointwise_indexed")
        else:
            _check(lib.emmy_pointwise(in_ptrs, in_dts, len(ins), sc_ptrs, sc_dts, len(scs), imm,
                                      len(imms), prog, len(g["program"]), g["result_reg"],
                                      int(g["compute"] == "f64"), _ptr(T("out")),
                                      DT_CODE[g["out_dtype"]], g["n"], st), "emmy_pointwise")
        launches += 1
    elif fam == "pointwise_int":
        g = plan["pointwise"]
        ins, scs, imms = g["inputs"], g["scalars"], g["immediates"]
        in_ptrs = (_vp * max(1, len(ins)))(*[_ptr(tensors[n]) for n in ins])
        in_dts = (_int * max(1, len(ins)))(*[DT_CODE[plan["tensors"][n]["dtype"]] for n in ins])
        sc_ptrs = (_vp * max(1, len(scs)))(*[_ptr(tensors[n]) for n in scs])
        sc_dts = (_int * max(1, len(scs)))(*[DT_CODE[plan["tensors"][n]["dtype"]] for n in scs])
        imm = (ctypes.c_int64 * max(1, len(imms)))(*[int(v) for v in imms])
        flat = [int(x) for row in g["program"] for x in row]
        prog = (_int * len(flat))(*flat)
        idx_arr = None
        if "input_index" in g:
            idx = []
            for n, (d, m) in zip(ins, g["input_index"]):
                idx += [int(d), int(m), tensors[n].numel()]
            idx_arr = (ctypes.c_int64 * len(idx))(*idx)
        _check(lib.emmy_pointwise_int(in_ptrs, in_dts, idx_arr, len(ins), sc_ptrs, sc_dts, len(scs),
                                      imm, len(imms), prog, len(g["program"]), g["result_reg"],
                                      _ptr(T("out")), DT_CODE[g["out_dtype"]],
                                      int(g.get("first", 0)), g["n"], int(g.get("value_bits", 64)),
                                      st), "emmy_pointwise_int")
        launches += 1
    else:
        raise ValueError(f"plan family {fam!r} has no launcher")
    return launches


_PIPE = {}


def _pipe_streams(device):
    """The upload, kernel and download streams ``Executor.run_pipelined`` uses on ``device``."""
    import torch
    key = torch.device(device).index
    if key not in _PIPE:
        _PIPE[key] = tuple(torch.cuda.Stream(device=device) for _ in range(3))
    return _PIPE[key]


class Executor:
    """Device buffers for one plan, reused across calls (H2D -> kernel -> D2H)."""

    def __init__(self, plan: dict, device=None):
        import torch
        self.plan = plan
        self.device = torch.device(device or "cuda")
        self.tensors = {}
        for name, spec in plan["tensors"].items():
            numel = math.prod(spec["shape"]) if spec["shape"] else 1
            self.tensors[name] = torch.empty(numel, dtype=torch_dtype(spec["dtype"]),
                                             device=self.device)
        nb = workspace_bytes(plan)
        self.workspace = torch.empty(nb, dtype=torch.uint8, device=self.device) if nb else None

    def upload(self, host: dict, stream=None) -> int:
        """Copy host arrays/tensors (pinned for true async) into the device buffers; returns bytes."""
        import torch
        nbytes = 0
        for name, arr in host.items():
            src = arr if isinstance(arr, torch.Tensor) else torch.from_numpy(arr)
            dst = self.tensors[name]
            dst.copy_(src.reshape(-1), non_blocking=True)
            nbytes += dst.numel() * dst.element_size()
        return nbytes

    def launch(self, stream=None) -> int:
        return run(self.plan, self.tensors, stream=stream, workspace=self.workspace, check=False)

    def inputs(self) -> list:
        """Plan tensors the kernels read.

        Outputs are written whole (or zeroed first, ``zero_outputs``) and are
        not read -- except the C of a split-K matmul whose atomic partial sums
        add onto what C already holds (``gemm.accumulate``).
        """
        outs = set(self.plan["outputs"])
        if self.plan.get("gemm", {}).get("accumulate"):
            outs.discard(self.plan["args"]["c"])
        return [n for n in self.plan["tensors"] if n not in outs]

    def run_pipelined(self, host: dict, out: dict, chunks: int | None = None, stream=None,
                      join: bool = True) -> int:
        """Host inputs in, host outputs out, with the copies overlapping the kernels.

        The plan is split into ``chunks`` independent sub-plans along its own
        shard axis (rows, batches, heads or element ranges, as ``ptxc.dist``
        shards it across GPUs).  Chunk i's inputs go up on one stream while
        chunk i-1 computes on a second and chunk i-2's outputs come down on a
        third, so both PCIe directions and the kernels run at once; tensors
        every chunk reads whole (weights, scalars) go up once, first.  Outputs
        are written whole by the kernels and never uploaded.  ``chunks``
        defaults to one per ~32 MiB of input.  ``host``/``out`` tensors should
        be pinned for the copies to be asynchronous.

        Ordered after ``stream`` (default: the current stream).  The three
        streams are shared by every Executor on the device, so consecutive
        calls with ``join=False`` queue behind one another without a stall;
        the last call of a step passes ``join=True`` (the default), which makes
        ``stream`` wait for every download.  Returns the library launches.
        """
        import torch
        from .dist import shard_plan
        cur = stream if stream is not None else torch.cuda.current_stream(self.device)
        s_in, s_k, s_out = _pipe_streams(self.device)
        outs = set(self.plan["outputs"])
        ins = self.inputs()
        if chunks is None:
            in_bytes = sum(self.tensors[n].numel() * self.tensors[n].element_size() for n in ins)
            chunks = max(1, min(64, -(-in_bytes // (32 << 20))))
        try:
            subs = [shard_plan(self.plan, i, chunks) for i in range(chunks)] if chunks > 1 else None
        except ValueError:
            subs = None
        if subs is None:
            subs = [(self.plan, {n: (0, t.numel()) for n, t in self.tensors.items()})]
        full = {n for n in ins if all(sl[n] == (0, self.tensors[n].numel()) for _, sl in subs)}
        for s in (s_in, s_k, s_out):
            s.wait_stream(cur)
        flat = {n: torch.as_tensor(host[n]).reshape(-1) for n in ins}
        launches = 0
        with torch.cuda.stream(s_in):
            for n in full:
                self.tensors[n].copy_(flat[n], non_blocking=True)
        for sub, sl in subs:
            with torch.cuda.stream(s_in):
                for n in ins:
                    if n not in full:
                        off, cnt = sl[n]
                        self.tensors[n][off:off + cnt].copy_(flat[n][off:off + cnt],
                                                             non_blocking=True)
                ev_in = torch.cuda.Event()
                ev_in.record(s_in)
            s_k.wait_event(ev_in)
            views = {n: self.tensors[n][sl[n][0]:sl[n][0] + sl[n][1]] for n in self.plan["tensors"]}
            launches += run(sub, views, stream=s_k, workspace=self.workspace, check=False)
            ev_k = torch.cuda.Event()
            ev_k.record(s_k)
            s_out.wait_event(ev_k)
            with torch.cuda.stream(s_out):
                for n in outs:
                    if n in out:
                        off, cnt = sl[n]
                        out[n].reshape(-1)[off:off + cnt].copy_(self.tensors[n][off:off + cnt],
                                                                non_blocking=True)
        if join:
            cur.wait_stream(s_out)
        return launches

    def download(self, names=None, out=None) -> dict:
        names = list(names or self.plan["outputs"])
        res = {}
        for name in names:
            if out is not None and name in out:
                out[name].copy_(self.tensors[name], non_blocking=True)
                res[name] = out[name]
            else:
                res[name] = self.tensors[name].cpu()
        return res


def run_host(plan: dict, host: dict) -> dict:
    """Convenience: numpy inputs in, numpy outputs out (zero-initialised outputs)."""
    import numpy as np
    import torch
    ex = Executor(plan)
    for name, t in ex.tensors.items():
        if name not in host:
            t.zero_()
    ex.upload({k: np.ascontiguousarray(v) for k, v in host.items()})
    ex.launch()
    torch.cuda.synchronize()
    return {k: v.numpy() for k, v in ex.download().items()}
