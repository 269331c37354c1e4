"""The committed reference goldens (``tests/golden``) and the fixture replicas.

* ``goldens.json`` / ``goldens.npz`` hold what the reference's own fixtures
  expect; where the reference checkout is present they are checked against
  it value for value.
* Each replica declares exactly the fixture's arguments (so the seeded inputs
  are the reference harness's), compiles to the same launch plan as the
  fixture's own IR, and the CPU oracle run on it reproduces the golden within
  the fixture's rtol/atol.  The GPU tests use the same replicas.
"""

from __future__ import annotations

import json

import numpy as np
import pytest

from conftest import REFERENCE_VARIANTS, load_variant, needs_reference, reference_variants
from golden import replicas
from oracle.interp import make_inputs, run_ir
from ptxc import Lowerer


def test_table_has_every_fixture_once():
    t = replicas.table()
    assert len(t) == 46
    for fid, e in t.items():
        exp, idx, _ = replicas.golden(fid)
        n = int(np.prod(e["shape"])) if e["shape"] else 1
        assert (idx is None and exp.size == n) or (idx is not None and idx.max() < n), fid


@needs_reference
def test_table_matches_reference_files():
    names = {p.name for p in reference_variants()}
    assert names == set(replicas.table())
    for fid in sorted(names):
        meta = json.loads((REFERENCE_VARIANTS / fid / "meta.json").read_text())
        full = np.load(REFERENCE_VARIANTS / fid / "expected.npz")[meta["graph_outputs"][0]]
        exp, idx, e = replicas.golden(fid)
        flat = full.reshape(-1)
        assert np.array_equal(flat if idx is None else flat[idx], exp), fid
        assert e["rtol"] == meta["rtol"] and e["atol"] == meta["atol"]


@pytest.mark.parametrize("fid", replicas.replica_ids())
def test_replica_declares_fixture_inputs(fid):
    _, meta, names = replicas.build(fid)
    assert replicas.same_inputs(fid, meta, names)


def test_every_fixture_has_a_replica():
    assert replicas.replica_ids() == sorted(replicas.table())


@pytest.mark.parametrize("fid", replicas.replica_ids())
def test_oracle_on_replica_reproduces_golden(fid):
    kop, meta, names = replicas.build(fid)
    host = replicas.fixture_inputs(fid, meta, names)
    out_name = next(a["name"] for a in meta["args"] if a.get("output"))
    out = run_ir(kop, meta, host)[out_name]
    worst, msg = replicas.compare(fid, out)
    assert worst <= 0, msg


def _plan_key(plan):
    fam = plan["family"]
    if fam == "pointwise":
        return plan["pointwise"]
    if fam in ("reduce", "rownorm", "softmax", "matvec"):
        return plan["view"], plan.get("params")
    if fam.startswith("gemm"):
        g = plan["gemm"]
        return {k: g[k] for k in ("batch", "m", "n", "k", "epilogue")}
    if fam.startswith("attention"):
        return plan["attention"]
    return None


@needs_reference
@pytest.mark.parametrize("fid", replicas.replica_ids())
def test_replica_plans_like_the_fixture(fid):
    kop, meta, _ = replicas.build(fid)
    mine = Lowerer(kop, meta).plan()
    fkop, fmeta, _ = load_variant(REFERENCE_VARIANTS / fid)
    theirs = Lowerer(fkop, fmeta["kernels"][-1]).plan()
    assert mine["family"] == theirs["family"]
    assert _plan_key(mine) == _plan_key(theirs)
