"""Emit the reference compiler's own PTX for every reference fixture and the
benchmark configurations (test infrastructure; run where the reference
checkout exists).

The reference is a Python compiler whose only missing piece is the
``emmy-ml`` package (``requirements.txt:1``); ``oracle/emmy_shim`` supplies the
``emmy`` modules it imports on top of this repository's IR classes.  The
reference's ``compile.py`` then runs **unmodified** as a subprocess, one
kernel package per call (``compile.py:70-106``), and its PTX (``.target sm_89``
by default, ``ptxc/lower.py:599``; the driver JIT-compiles it for sm_100) is
written with the package's ``meta.json`` into ``oracle/_ref/<name>/``.  That
directory is git-ignored and travels to the GPU box, where
``oracle/ref_ptx.py`` loads and launches the PTX exactly as the reference
harness does (``tools/localrun.py:102-142``).

Usage: ``python oracle/make_ref_ptx.py [REFERENCE_DIR]``; without the argument
the checkout is found by ``oracle/refdir.py`` (``EMMY_REFERENCE_DIR``, else a
``reference`` checkout beside this repository).  The test set-up
(``tests/conftest.py``) runs it when ``oracle/_ref`` is missing or older than
this file.
"""

from __future__ import annotations

import json
import os
import shutil
import subprocess
import sys
import tempfile
from pathlib import Path

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
PKG = ROOT / "emmy-ptx-compiler-submission_b200"
OUT = HERE / "_ref"

# benchmark configurations (the bench's family cases) as synthesised IR
BENCH_CASES = {
    "K1_rmsnorm": lambda s: s.rmsnorm(4096, 512, eps=1e-6),
    "K2a_softmax": lambda s: s.softmax([32, 16, 512, 512]),
    "K2b_layernorm": lambda s: s.layernorm(16384, 1024),
    "K4b_matvec_f64": lambda s: s.matvec(16384, 16384),
    "K4a_splitk_f32": lambda s: s.matmul(256, 256, 65536, splits=64, tm=128, tn=128, rm=8, rn=8),
    "K3a_gemm_f16": lambda s: s.matmul(4096, 8192, 2048, dtype="f16", out_dtype="f16", bias=True,
                                       relu=True, tm=128, tn=128, rm=8, rn=8),
    "K3b_bmm_f16": lambda s: s.matmul(512, 512, 512, batch=64, dtype="f16", out_dtype="f16",
                                      tm=128, tn=128, rm=8, rn=8),
    "K5_attention_f16": lambda s: s.attention(8, 32, 512, 128, dtype="f16"),
    "F8a_pointwise_add": lambda s: s.pointwise(1 << 26, ("add", "x0", "x1"), "f32"),
    "F8d_pointwise_int": lambda s: s.pointwise(1 << 26, ("add", "x0", "x1"), "i32"),
}

# integer pointwise programs (the reference's integer Assign path): each one
# assembles with ptxas for sm_100a; shifts and copies of 8/16-bit values do
# not (the reference passes an s64 shift count where PTX wants .u32, and a
# 32-bit register to mov.u16), so they are left out here
_NZ = ("where", ("equal", "x1", ("imm", 0)), ("imm", 7), "x1")     # a divisor that is never 0
INT_CASES = {
    "I_add_i32": lambda s: s.pointwise(4099, ("add", "x0", "x1"), "i32"),
    "I_mul_imm_u8": lambda s: s.pointwise(4099, ("multiply", "x0", ("imm", 3)), "u8"),
    "I_div_i64": lambda s: s.pointwise(4099, ("divide", "x0", _NZ), "i64"),
    "I_rem_i16": lambda s: s.pointwise(4099, ("remainder", "x0", _NZ), "i16"),
    "I_div_u32": lambda s: s.pointwise(4099, ("floor_divide", "x0", _NZ), "u32"),
    "I_xor_sub_u32": lambda s: s.pointwise(4099, ("subtract", ("bitwise_xor", "x0", "x1"), "x1"),
                                           "u32"),
    "I_max_min_u64": lambda s: s.pointwise(4099, ("minimum", ("maximum", "x0", "x1"), "x0"), "u64"),
    "I_where_cmp_i32": lambda s: s.pointwise(
        4099, ("where", ("greater", "x0", "x1"), "x0", ("imm", -7)), "i32"),
    "I_and_or_i8": lambda s: s.pointwise(
        4099, ("where", ("bitwise_or", ("bitwise_and", "x0", "x1"), ("less", "x0", ("imm", 0))),
               "x0", "x1"), "i8"),
    "I_i32_to_f32": lambda s: s.pointwise(4099, ("add", "x0", "x1"), "i32", out_dtype="f32"),
    "I_i64_to_f16": lambda s: s.pointwise(
        4099, ("multiply", "x0", "x1"), "i64", out_dtype="f16",
        inits={"x0": {"dist": "int", "low": -300, "high": 300},
               "x1": {"dist": "int", "low": -300, "high": 300}}),
    "I_u16_to_f64": lambda s: s.pointwise(4099, ("add", "x0", ("imm", 1)), "u16", out_dtype="f64"),
    "I_float_in_i32": lambda s: s.pointwise(
        4099, ("add", "x0", "x1"), "i32", dtypes={"x1": "f32"},
        inits={"x1": {"dist": "uniform", "low": -1e9, "high": 1e9}}),
    "I_f16_f64_in_i64": lambda s: s.pointwise(
        4099, ("subtract", "x0", "x1"), "i64", dtypes={"x0": "f16", "x1": "f64"},
        inits={"x0": {"dist": "normal", "std": 300.0}, "x1": {"dist": "normal", "std": 1e12}}),
    "I_const_i8": lambda s: s.pointwise(4099, ("subtract", "x0", ("const", "c", -5)), "i8"),
    "I_chain_mixed": lambda s: s.pointwise(
        4099, ("add", ("multiply", "x0", "x1"), ("remainder", "x0", _NZ)), "i32",
        dtypes={"x0": "u8", "x1": "i16"}, out_dtype="i16"),
}


def _compile(ref: Path, ir_path: Path):
    env = dict(os.environ)
    env["PYTHONPATH"] = os.pathsep.join([str(ref), str(HERE / "emmy_shim"), str(PKG)])
    r = subprocess.run([sys.executable, str(ref / "compile.py"), str(ir_path)], env=env,
                       capture_output=True, text=True, timeout=600)
    return r.returncode, r.stdout, r.stderr.strip()


def main(ref: Path) -> int:
    sys.path[:0] = [str(PKG)]
    from emmy_ir import synth
    from emmy_ir.serialize import write_package
    OUT.mkdir(exist_ok=True)
    jobs = []
    for d in sorted(p for p in (ref / "tests" / "variants").iterdir() if (p / "meta.json").exists()):
        jobs.append((d.name, next(d.glob("*.ir.json")), d / "meta.json"))
    tmp = Path(tempfile.mkdtemp(prefix="emmy_ref_"))
    for name, make in {**BENCH_CASES, **INT_CASES}.items():
        kop, meta = make(synth)
        ir = write_package(tmp / name, kop, meta)
        jobs.append((name, ir, tmp / name / "meta.json"))
    report = {}
    for name, ir, meta in jobs:
        rc, ptx, err = _compile(ref, ir)
        dst = OUT / name
        if dst.exists():
            shutil.rmtree(dst)
        dst.mkdir()
        shutil.copy(meta, dst / "meta.json")
        if rc == 0:
            (dst / "kernel.ptx").write_text(ptx)
        report[name] = {"rc": rc, "error": err.splitlines()[-1] if err else ""}
        print(f"{name}: rc {rc} {report[name]['error']}")
    (OUT / "report.json").write_text(json.dumps(report, indent=1, sort_keys=True) + "\n")
    shutil.rmtree(tmp, ignore_errors=True)
    return 0


if __name__ == "__main__":
    if len(sys.argv) > 1:
        _ref = Path(sys.argv[1])
    else:
        sys.path.insert(0, str(ROOT))
        from oracle.refdir import reference_dir
        _ref = reference_dir()
        if _ref is None:
            sys.exit("make_ref_ptx: no reference checkout (set EMMY_REFERENCE_DIR)")
    sys.exit(main(_ref))
