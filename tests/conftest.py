"""Shared test set-up: import paths, the ``gpu`` marker, fixture locations.

``-m "not gpu"`` runs everywhere (no GPU needed).  ``-m gpu`` needs a B200 and
the built ``libemmyb200.so``; those tests call the kernels through the C-ABI.
"""

from __future__ import annotations

import json
import os
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
PKG = ROOT / "emmy-ptx-compiler-submission_b200"
for p in (str(ROOT), str(PKG)):
    if p not in sys.path:
        sys.path.insert(0, p)

from oracle.refdir import reference_dir  # noqa: E402
from oracle.refdir import reference_variants as _variants_dir  # noqa: E402

# The reference's own fixture packages, read in place when a reference checkout
# is available (``EMMY_REFERENCE_DIR``, else a ``reference`` checkout beside
# this repository; they are not redistributable, so nothing is copied).  On a
# machine without one (a GPU box) the tests that need it are skipped.
REFERENCE_VARIANTS = _variants_dir() or ROOT / "_no_reference_checkout"


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and libemmyb200.so")
    config.addinivalue_line("markers", "slow: long CPU oracle runs")


def pytest_sessionstart(session):
    """Test set-up: the reference compiler's own PTX for the GPU comparisons.

    ``oracle/make_ref_ptx.py`` runs the unmodified reference compiler over its
    fixtures and the benchmark configurations into ``oracle/_ref`` (which then
    travels to the GPU box).  It runs here when a reference checkout exists and
    ``oracle/_ref`` is missing or older than the generator; elsewhere the
    files already present are used, and the tests that need them skip
    without them.
    """
    ref = reference_dir()
    if ref is None or os.environ.get("EMMY_SKIP_REF_PTX"):
        return
    gen = ROOT / "oracle" / "make_ref_ptx.py"
    report = ROOT / "oracle" / "_ref" / "report.json"
    if report.exists() and report.stat().st_mtime >= gen.stat().st_mtime:
        return
    import subprocess
    subprocess.run([sys.executable, str(gen), str(ref)], check=False, capture_output=True,
                   timeout=1800)


def reference_variants():
    if not REFERENCE_VARIANTS.is_dir():
        return []
    return sorted(p for p in REFERENCE_VARIANTS.iterdir() if (p / "meta.json").exists())


def load_variant(path: Path):
    from emmy_ir import Graph
    meta = json.loads((path / "meta.json").read_text())
    ir = next(path.glob("*.ir.json"))
    g = Graph.from_dict(json.loads(ir.read_text()))
    kop = [n.op for n in g.nodes.values() if type(n.op).__name__ == "KernelOp"][0]
    return kop, meta, ir


needs_reference = pytest.mark.skipif(not REFERENCE_VARIANTS.is_dir(),
                                     reason="reference fixtures not present on this machine")
