"""Run the reference compiler's own PTX on the GPU (test infrastructure only).

``oracle/make_ref_ptx.py`` writes ``oracle/_ref/<name>/{kernel.ptx, meta.json}``
with the unmodified reference compiler.  ``RefKernel`` loads that PTX through
the CUDA driver (the driver JIT-compiles the ``sm_89`` PTX for the B200) and
launches it the way the reference harness does (``tools/localrun.py:102-142``):
one u64 device pointer per argument in ``arg_order``, the meta.json grid,
block and dynamic shared memory, outputs zero-filled first (the harness
allocates them with ``np.zeros``; ``zero_outputs`` needs nothing more).

It is the GPU-side oracle ("the reference's own emitted-PTX kernels") and the
reference timing beside the B200 kernels; nothing in the product imports it.
"""

from __future__ import annotations

import ctypes
import json
import math
from pathlib import Path

HERE = Path(__file__).resolve().parent
REF_DIR = HERE / "_ref"

_CU = None


def _cuda():
    global _CU
    if _CU is None:
        _CU = ctypes.CDLL("libcuda.so.1")
    return _CU


def _check(rc, what):
    if rc != 0:
        msg = ctypes.c_char_p()
        _cuda().cuGetErrorString(rc, ctypes.byref(msg))
        raise RuntimeError(f"{what}: CUDA driver error {rc} ({(msg.value or b'').decode()})")


def available(name: str) -> bool:
    return (REF_DIR / name / "kernel.ptx").exists()


def names() -> list:
    if not REF_DIR.is_dir():
        return []
    return sorted(p.name for p in REF_DIR.iterdir() if (p / "kernel.ptx").exists())


class RefKernel:
    """One reference PTX entry, loaded into the current CUDA context."""

    def __init__(self, name: str):
        import torch
        torch.cuda.init()
        torch.zeros(1, device="cuda")                      # make the primary context current
        d = REF_DIR / name
        self.meta_pkg = json.loads((d / "meta.json").read_text())
        self.k = self.meta_pkg["kernels"][-1]
        ptx = (d / "kernel.ptx").read_bytes() + b"\0"
        cu = _cuda()
        self._mod = ctypes.c_void_p()
        _check(cu.cuModuleLoadData(ctypes.byref(self._mod), ctypes.c_char_p(ptx)), "cuModuleLoadData")
        self._fn = ctypes.c_void_p()
        _check(cu.cuModuleGetFunction(ctypes.byref(self._fn), self._mod, self.k["entry"].encode()),
               "cuModuleGetFunction")
        self.smem = int(self.k.get("smem_bytes", 0))
        if self.smem > 48 * 1024:
            # CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES
            _check(cu.cuFuncSetAttribute(self._fn, 8, ctypes.c_int(self.smem)), "cuFuncSetAttribute")

    @property
    def args(self) -> list:
        return self.k["args"]

    def alloc(self, host: dict, device="cuda") -> dict:
        """Device tensors for every argument (host arrays by name; outputs zero)."""
        import numpy as np
        import torch
        out = {}
        for a in self.k["args"]:
            n = math.prod(a["shape"]) if a["shape"] else 1
            dt = {"f32": torch.float32, "f16": torch.float16, "f64": torch.float64,
                  "i8": torch.int8, "u8": torch.uint8, "i16": torch.int16, "u16": torch.uint16,
                  "i32": torch.int32, "u32": torch.uint32, "i64": torch.int64,
                  "u64": torch.uint64}[a["dtype"]]
            if a.get("output"):
                out[a["name"]] = torch.zeros(n, dtype=dt, device=device)
            else:
                out[a["name"]] = torch.from_numpy(np.ascontiguousarray(host[a["name"]]).reshape(-1)).to(device)
        return out

    def launch(self, tensors: dict, stream=None) -> None:
        import torch
        order = self.k.get("arg_order") or [a["name"] for a in self.k["args"]]
        vals = [ctypes.c_uint64(tensors[n].data_ptr()) for n in order]
        params = (ctypes.c_void_p * len(vals))(*[ctypes.addressof(v) for v in vals])
        st = stream if stream is not None else torch.cuda.current_stream()
        g, b = self.k["grid"], self.k["block"]
        _check(_cuda().cuLaunchKernel(self._fn, g[0], g[1], g[2], b[0], b[1], b[2], self.smem,
                                      ctypes.c_void_p(st.cuda_stream), params, None),
               "cuLaunchKernel")

    def run(self, host: dict) -> dict:
        """Allocate, launch once, synchronise; returns every buffer as numpy."""
        import torch
        t = self.alloc(host)
        for a in self.k["args"]:
            if a.get("output"):
                t[a["name"]].zero_()
        self.launch(t)
        torch.cuda.synchronize()
        return {k: v.cpu().numpy() for k, v in t.items()}

    def close(self):
        if self._mod:
            _cuda().cuModuleUnload(self._mod)
            self._mod = ctypes.c_void_p()
