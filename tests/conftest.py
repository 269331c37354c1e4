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

# The reference's own fixture packages, read in place when this machine has
# the reference checkout (they are not redistributable, so nothing is copied).
REFERENCE_VARIANTS = Path(os.environ.get("EMMY_REFERENCE_VARIANTS",
                                         "/root/reference/tests/variants"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and libemmyb200.so")
    config.addinivalue_line("markers", "slow: long CPU oracle runs")


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
