"""GPU parity against the reference's own goldens, every fixture.

Each of the reference's 46 fixture kernels is rebuilt with the synthesiser
(``tests/golden/replicas.py``: same statement shape, the fixture's seeded
inputs), compiled to a plan, run through ``libemmyb200.so`` and compared with
the stored expected output (``tests/golden/goldens.npz``) using the fixture's
own rtol/atol: ``|got - want| <= atol + rtol * |want|`` at every stored
position (all of them up to 8192 elements, 2048 evenly spaced ones beyond).
No reference checkout is needed on the GPU box.
"""

from __future__ import annotations

import pytest

from golden import replicas
from gpu_util import run_on_gpu

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("fid", replicas.replica_ids())
def test_kernel_reproduces_reference_golden(fid):
    kop, meta, names = replicas.build(fid)
    out_name = next(a["name"] for a in meta["args"] if a.get("output"))
    plan, _, out = run_on_gpu(kop, meta, replicas.fixture_inputs(fid, meta, names))
    worst, msg = replicas.compare(fid, out[out_name])
    assert worst <= 0, f"{plan['family']}: {msg}"
