"""Build recipe for libemmyb200.so: every ``csrc/*.cu`` compiled for sm_100a.

``python build.py`` (or ``build()`` from Python) runs nvcc once per source
file in parallel and links the objects into ``libemmyb200.so`` next to this
file.  Objects go to ``_build/``; both are git-ignored.  Nothing here needs a
GPU: nvcc cross-compiles for ``sm_100a``.
"""

from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
OUT = HERE / "libemmyb200.so"
BUILD = HERE / "_build"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-O2",
    "-diag-suppress", "177",
    "-I", str(HERE.parent / "include"),
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found; set NVCC")


def _stale(src: Path, obj: Path) -> bool:
    if not obj.exists():
        return True
    deps = [src] + sorted(CSRC.glob("*.cuh")) + [HERE.parent / "include" / "emmy_b200.h"]
    return any(d.stat().st_mtime > obj.stat().st_mtime for d in deps if d.exists())


def build(verbose: bool = False, force: bool = False) -> Path:
    nvcc = _nvcc()
    BUILD.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    jobs = []
    for src in sources:
        obj = BUILD / (src.stem + ".o")
        if force or _stale(src, obj):
            jobs.append((src, obj))

    def compile_one(job):
        src, obj = job
        cmd = [nvcc, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode:
            raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
        if verbose and (r.stdout or r.stderr):
            print(r.stdout + r.stderr, file=sys.stderr)
        return obj

    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        list(ex.map(compile_one, jobs))
    objs = [BUILD / (s.stem + ".o") for s in sources]
    if jobs or not OUT.exists() or any(o.stat().st_mtime > OUT.stat().st_mtime for o in objs):
        tmp = OUT.with_suffix(".so.tmp")
        cmd = [nvcc, "-shared", "-gencode", "arch=compute_100a,code=sm_100a",
               *[str(o) for o in objs], "-o", str(tmp)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, OUT)
    return OUT


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv, force="-f" in sys.argv))
