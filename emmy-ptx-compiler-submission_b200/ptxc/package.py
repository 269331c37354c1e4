"""Problem packages with several kernels: one meta.json, kernels run in order.

The reference harness (``tools/localrun.py:150-200``, ``tools/prof.py:55-90``)
reads ``meta.json["kernels"]``, compiles each entry's ``<entry>.ir.json``
(``tools/irfiles.py:17-29``: the exact file, else the package's only IR file,
else an error naming what it found), and launches the kernels in order.  An
argument marked ``"intermediate"`` takes the values an earlier kernel wrote
under that name (converted to this argument's dtype); outputs start at zero;
a kernel with ``"final": false`` produces values for later kernels only.  The
matmul + bias + ReLU problem is such a chain: a matmul kernel, then an
elementwise kernel reading the product and a broadcast bias
(``docs/COVERAGE.md:55,97``: ``adv_mm_bias_relu``, ``k_relu__partial`` ->
``k_relu``).

``Chain`` compiles every kernel to a launch plan.  ``ChainExecutor`` keeps
every tensor of the chain in device memory -- an intermediate never leaves the
GPU -- and runs the plans on one stream.  With ``fuse=True`` (the default) a
matmul whose product feeds only a following bias / ReLU elementwise kernel is
run as one matmul with that epilogue (``fuse_gemm_epilogue``): the product is
never written to HBM or read back.  Fusion is applied only where the fused
epilogue gives the same bits as the two kernels (rules in
``fuse_gemm_epilogue``).
"""

from __future__ import annotations

import copy
import json
import math
from pathlib import Path

from .common import CompileError
from .lower import Lowerer
from .match_pointwise import ARITY, OPCODES, UNARY


class IRError(Exception):
    """No IR file for a kernel entry (the reference's ``tools/irfiles.py:13``)."""


def resolve_ir(problem_dir, entry: str) -> Path:
    """``<entry>.ir.json`` in the package, else its only IR file, else IRError.

    An exact name is required when there are several files: entries such as
    ``k_sum_1`` and ``k_sum_1__partial`` share a prefix (``tools/irfiles.py:17-29``).
    """
    pdir = Path(problem_dir)
    exact = pdir / f"{entry}.ir.json"
    if exact.is_file():
        return exact
    found = sorted(pdir.glob("*.ir.json"))
    if len(found) == 1:
        return found[0]
    if not found:
        raise IRError(f"{pdir}: no .ir.json files")
    raise IRError(f"{pdir}: no IR for entry {entry!r}; found " + ", ".join(p.name for p in found))


def _kernel_op(ir_path: Path, entry: str):
    from emmy_ir.graph import Graph
    try:
        graph = Graph.from_dict(json.loads(ir_path.read_text()))
    except (ValueError, TypeError, KeyError, SyntaxError, NameError) as exc:
        raise CompileError(f"invalid IR in {ir_path.name}: {exc}") from exc
    ops = [n.op for n in graph.nodes.values() if type(n.op).__name__ == "KernelOp"]
    if len(ops) != 1:
        raise CompileError(f"{ir_path.name}: expected exactly one KernelOp, found {len(ops)}")
    if ops[0].name != entry:
        raise CompileError(f"{ir_path.name}: KernelOp {ops[0].name!r} is not entry {entry!r}")
    return ops[0]


class Chain:
    """The kernels of one package, compiled, in launch order."""

    def __init__(self, steps: list, meta: dict | None = None):
        # step: {"entry", "meta" (the kernel's meta.json entry), "plan", "final"}
        self.steps = steps
        self.meta = meta or {}

    @classmethod
    def load(cls, problem_dir) -> "Chain":
        pdir = Path(problem_dir)
        meta = json.loads((pdir / "meta.json").read_text())
        kernels = meta.get("kernels") or []
        if not kernels:
            raise CompileError(f"{pdir / 'meta.json'}: no kernels")
        steps = []
        for k in kernels:
            kop = _kernel_op(resolve_ir(pdir, k["entry"]), k["entry"])
            steps.append(cls._step(kop, k))
        return cls(steps, meta)

    @classmethod
    def from_kernels(cls, pairs) -> "Chain":
        """From ``(KernelOp, meta kernel entry)`` pairs (synthesised packages)."""
        return cls([cls._step(kop, k) for kop, k in pairs])

    @staticmethod
    def _step(kop, k):
        return {"entry": k["entry"], "meta": k, "plan": Lowerer(kop, k).plan(),
                "final": bool(k.get("final", True))}

    def tensors(self) -> dict:
        """Every tensor name of the chain -> (dtype, numel) of its first declaration."""
        out = {}
        for st in self.steps:
            for a in st["meta"]["args"]:
                out.setdefault(a["name"], (a["dtype"], math.prod(a["shape"]) if a["shape"] else 1))
        return out

    def host_inputs(self) -> list:
        """Arguments the caller provides: neither written by a kernel nor intermediate."""
        written = set()
        need = []
        for st in self.steps:
            for a in st["meta"]["args"]:
                if a.get("output"):
                    written.add(a["name"])
                elif not a.get("intermediate") and a["name"] not in written \
                        and a["name"] not in need:
                    need.append(a["name"])
        return need

    def outputs(self) -> list:
        """Outputs of the kernels marked final (the values a package is checked on)."""
        out = []
        for st in self.steps:
            if st["final"]:
                out += [a["name"] for a in st["meta"]["args"]
                        if a.get("output") and a["name"] not in out]
        return out


def _pointwise_form(g: dict):
    """The program of a pointwise plan as a tree over its registers."""
    ni, ns, nm = len(g["inputs"]), len(g["scalars"]), len(g["immediates"])
    names = {v: k for k, v in OPCODES.items()}
    regs = {}
    for i in range(ni):
        regs[i] = ("in", i)
    for i in range(ns):
        regs[ni + i] = ("scalar", i)
    for i in range(nm):
        regs[ni + ns + i] = ("imm", float(g["immediates"][i]))
    for op, dst, a, b, c in g["program"]:
        nm_ = names[op]
        arity = ARITY.get(nm_, 1 if nm_ in UNARY else 2)
        regs[dst] = (nm_,) + tuple(regs[r] for r in (a, b, c)[:arity])
    return regs[g["result_reg"]]


def _epilogue_of(form, x_reg: int, bias_reg):
    """(epilogue bits, rounds the sum to f16) when ``form`` is x [+ bias] [relu]."""
    rounded = False

    def strip(f):
        nonlocal rounded
        while f[0] in ("round_f16", "copy"):
            rounded = rounded or f[0] == "round_f16"
            f = f[1]
        return f

    f = strip(form)
    relu = False
    if f[0] == "relu":
        relu, f = True, strip(f[1])
    elif f[0] == "maximum" and ("imm", 0.0) in f[1:]:
        other = f[1] if f[2] == ("imm", 0.0) else f[2]
        relu, f = True, strip(other)
    x = ("in", x_reg)
    if f == x:
        return (2 if relu else 0), rounded, False
    if bias_reg is not None and f[0] == "add" and set(f[1:]) == {x, ("in", bias_reg)}:
        return (1 | (2 if relu else 0)), rounded, True
    return None


def fuse_gemm_epilogue(gemm: dict, pw: dict, gemm_out_final: bool):
    """One matmul plan doing ``gemm`` then the elementwise ``pw`` step, or None.

    Fused when, bit for bit, the matmul epilogue (round the product to the
    intermediate's dtype, + bias[n] in f32, ReLU, convert to the output
    dtype) computes what the two kernels do:

    * ``gemm`` writes C whole (no split-K atomics, no epilogue of its own) and
      C is needed only by ``pw`` (not a final output);
    * ``pw`` reads C contiguously at the element it writes, at most one other
      tensor -- an f32 bias broadcast along rows (index ``e % N``) -- no
      scalar constants, and computes ``x``, ``x + bias``, ``relu(...)`` or
      ``maximum(..., 0)`` in f32;
    * C's dtype in ``pw`` is C's dtype in ``gemm``;
    * an f16 C is rounded first (``EMMY_EPI_ROUND_F16``, f16 matmul only);
      an f16 rounding of the sum inside ``pw`` is kept only when the output
      is f16 (rounding twice to f16 then equals rounding once);
    * the output dtype is one the matmul kernel writes (f32; f16 for f16
      operands).
    """
    if gemm_out_final or gemm["family"] not in ("gemm_f16", "gemm_f32") or pw["family"] != "pointwise":
        return None
    g, p = gemm["gemm"], pw["pointwise"]
    if g["epilogue"] or g["accumulate"] or g["splits"] != 1 or p["compute"] != "f32" or p["scalars"]:
        return None
    c = gemm["args"]["c"]
    cdt = gemm["tensors"][c]["dtype"]
    numel = g["batch"] * g["m"] * g["n"]
    if p["n"] != numel or c not in p["inputs"] or pw["tensors"][c]["dtype"] != cdt:
        return None
    index = p.get("input_index") or [[0, 0]] * len(p["inputs"])
    x_reg = p["inputs"].index(c)
    if index[x_reg] != [0, 0] or p["inputs"].count(c) != 1 or len(p["inputs"]) > 2:
        return None
    bias_reg = None
    if len(p["inputs"]) == 2:
        bias_reg = 1 - x_reg
        bname = p["inputs"][bias_reg]
        if index[bias_reg] != [1, g["n"]] or pw["tensors"][bname]["dtype"] != "f32" \
                or math.prod(pw["tensors"][bname]["shape"]) != g["n"]:
            return None
    got = _epilogue_of(_pointwise_form(p), x_reg, bias_reg)
    if got is None:
        return None
    epi, rounded, uses_bias = got
    if bias_reg is not None and not uses_bias:
        return None
    odt = p["out_dtype"]
    if rounded and odt != "f16":
        return None
    if gemm["family"] == "gemm_f32" and odt != "f32":
        return None
    if cdt == "f16":
        if gemm["family"] != "gemm_f16":
            return None
        epi |= 4                                  # EMMY_EPI_ROUND_F16
    out = pw["args"]["out"]
    fused = copy.deepcopy(gemm)
    fused["entry"] = gemm["entry"] + "+" + pw["entry"]
    fused["args"]["c"] = out
    fused["tensors"] = {k: v for k, v in fused["tensors"].items() if k != c}
    fused["tensors"][out] = dict(pw["tensors"][out])
    fused["outputs"] = [out]
    fused["zero_outputs"] = []
    fused["gemm"]["epilogue"] = epi
    if uses_bias:
        fused["args"]["bias"] = p["inputs"][bias_reg]
        fused["tensors"][p["inputs"][bias_reg]] = dict(pw["tensors"][p["inputs"][bias_reg]])
    if fused["family"] == "gemm_f16":
        fused["gemm"]["out_dtype"] = 1 if odt == "f16" else 0
    fused["dtypes"] = dict(fused.get("dtypes", {}), c=odt)
    fused["fused_from"] = [gemm["entry"], pw["entry"]]
    return fused


def _conversion_plan(name_src: str, src_dtype: str, name_dst: str, dst_dtype: str, n: int) -> dict:
    """A pointwise copy from one dtype to another (an intermediate re-typed by
    the kernel that reads it; the harness round-trips it through the host)."""
    return {
        "format": "emmy-b200-plan/1", "entry": f"convert_{name_src}",
        "arg_order": [name_src, name_dst],
        "tensors": {name_src: {"dtype": src_dtype, "shape": [n]},
                    name_dst: {"dtype": dst_dtype, "shape": [n]}},
        "outputs": [name_dst], "zero_outputs": [],
        "family": "pointwise", "symbol": "emmy_pointwise", "args": {"out": name_dst},
        "pointwise": {"n": n, "inputs": [name_src], "scalars": [], "immediates": [],
                      "program": [[0, 1, 0, 0, 0]], "result_reg": 1,
                      "compute": "f64" if "f64" in (src_dtype, dst_dtype) else "f32",
                      "out_dtype": dst_dtype},
        "params": {}, "dtypes": {"out": dst_dtype},
    }


def schedule(chain: Chain, fuse: bool = True) -> list:
    """The launch list: ``(plan, {plan tensor -> chain buffer})`` per launch.

    Chain buffers are named by tensor; an intermediate re-typed by its reader
    gets its own buffer ``name@dtype`` filled by a conversion launch.
    """
    dtype_of = {}                      # buffer -> dtype
    latest = {}                        # tensor name -> buffer holding its current values
    launches = []
    steps = chain.steps
    readers = {}                       # tensor -> indices of steps reading it as intermediate
    for i, st in enumerate(steps):
        for a in st["meta"]["args"]:
            if a.get("intermediate"):
                readers.setdefault(a["name"], []).append(i)
    i = 0
    while i < len(steps):
        st = steps[i]
        plan = st["plan"]
        if fuse and i + 1 < len(steps):
            nxt = steps[i + 1]
            c = plan.get("args", {}).get("c")
            inter = {a["name"] for a in nxt["meta"]["args"] if a.get("intermediate")}
            only_next = c in inter and readers.get(c) == [i + 1] and \
                not any(c == a["name"] for s in steps[i + 2:] for a in s["meta"]["args"])
            if only_next:
                fused = fuse_gemm_epilogue(plan, nxt["plan"], st["final"])
                if fused is not None:
                    bind = {n: n for n in fused["tensors"]}
                    for n in bind:
                        dtype_of.setdefault(n, fused["tensors"][n]["dtype"])
                    latest[fused["args"]["c"]] = fused["args"]["c"]
                    launches.append((fused, bind))
                    i += 2
                    continue
        bind = {}
        for a in st["meta"]["args"]:
            n = a["name"]
            if a.get("intermediate"):
                if n not in latest:
                    raise CompileError(f"{st['entry']}: intermediate {n!r} has no producer")
                src = latest[n]
                if dtype_of[src] != a["dtype"]:
                    conv = f"{n}@{a['dtype']}"
                    numel = math.prod(a["shape"]) if a["shape"] else 1
                    launches.append((_conversion_plan(src, dtype_of[src], conv, a["dtype"], numel),
                                     {src: src, conv: conv}))
                    dtype_of[conv] = a["dtype"]
                    src = conv
                bind[n] = src
            else:
                bind[n] = n
                dtype_of.setdefault(n, a["dtype"])
                if dtype_of[n] != a["dtype"]:
                    raise CompileError(f"{st['entry']}: {n!r} declared {a['dtype']} and {dtype_of[n]}")
        for a in st["meta"]["args"]:
            if a.get("output"):
                latest[a["name"]] = a["name"]
        launches.append((plan, bind))
        i += 1
    return launches


class ChainExecutor:
    """Device buffers for a whole chain; intermediates stay on the device."""

    def __init__(self, chain: Chain, device=None, fuse: bool = True):
        import torch
        from .launch import torch_dtype, workspace_bytes
        self.chain = chain
        self.device = torch.device(device or "cuda")
        self.launch_list = schedule(chain, fuse)
        self.buffers = {}
        for plan, bind in self.launch_list:
            for pname, buf in bind.items():
                spec = plan["tensors"][pname]
                numel = math.prod(spec["shape"]) if spec["shape"] else 1
                have = self.buffers.get(buf)
                if have is None:
                    self.buffers[buf] = torch.zeros(numel, dtype=torch_dtype(spec["dtype"]),
                                                    device=self.device)
                elif have.numel() != numel:
                    raise CompileError(f"{plan['entry']}: {pname!r} has {numel} elements, "
                                       f"the chain's buffer {have.numel()}")
        nb = max([workspace_bytes(p) for p, _ in self.launch_list] + [0])
        self.workspace = torch.empty(nb, dtype=torch.uint8, device=self.device) if nb else None

    @property
    def fused(self) -> list:
        return [p["fused_from"] for p, _ in self.launch_list if "fused_from" in p]

    def upload(self, host: dict) -> int:
        """Host values of the chain's inputs (by tensor name); returns bytes copied."""
        import torch
        nbytes = 0
        for name in self.chain.host_inputs():
            if name not in host or name not in self.buffers:
                continue
            src = host[name] if isinstance(host[name], torch.Tensor) else torch.from_numpy(host[name])
            dst = self.buffers[name]
            dst.copy_(src.reshape(-1), non_blocking=True)
            nbytes += dst.numel() * dst.element_size()
        return nbytes

    def launch(self, stream=None) -> int:
        from .launch import run
        launches = 0
        for plan, bind in self.launch_list:
            views = {pname: self.buffers[buf] for pname, buf in bind.items()}
            launches += run(plan, views, stream=stream, workspace=self.workspace, check=False)
        return launches

    def download(self, names=None) -> dict:
        names = names if names is not None else [n for n in self.chain.outputs() if n in self.buffers]
        return {n: self.buffers[n].cpu() for n in names}
