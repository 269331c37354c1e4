"""The shape catalogue (``emmy_ir.catalogue``): every catalogued problem shape
compiles to B200 plans, round-trips through a package on disk, and -- on the
GPU -- matches a float64 reference within the tolerance the reference checks
that problem with.  On the CPU the IR interpreter is held to the same
references for the entries it evaluates in well under a second.
"""

from __future__ import annotations

import numpy as np
import pytest

from catalogue_refs import REFS, check, final_output, host_inputs, shaped
from emmy_ir import catalogue
from oracle.interp import run_chain
from ptxc.package import Chain, schedule

IDS = catalogue.ids()


def test_every_entry_has_a_reference():
    assert set(IDS) == set(REFS)
    assert not set(catalogue.SKIPPED) & set(IDS)


@pytest.mark.parametrize("spec", IDS)
def test_entry_compiles(spec):
    chain = Chain.from_kernels(catalogue.build(spec))
    launches = schedule(chain)
    assert launches and all(p["family"] for p, _ in launches)


def test_packages_round_trip(tmp_path):
    for spec in ("adv_mm_gelu", "adv_mm_bias_relu", "dt_softmax16", "x_attn_s48_h96"):
        catalogue.write(spec, tmp_path / spec)
        chain = Chain.load(tmp_path / spec)
        assert [s["entry"] for s in chain.steps] == [k[1]["entry"] for k in catalogue.build(spec)]


def _small(spec):
    pairs = catalogue.build(spec)
    work = 0
    for _, meta in pairs:
        work += sum(int(np.prod(a["shape"])) for a in meta["args"])
    big_kinds = ("mm", "attn", "bmm")
    return work <= 300_000 and not any(k in spec for k in big_kinds)


@pytest.mark.parametrize("spec", [s for s in IDS if _small(s)])
def test_oracle_meets_the_reference(spec):
    pairs = catalogue.build(spec)
    host = host_inputs(pairs)
    got = run_chain(pairs, host)[final_output(pairs)]
    fn, rtol, atol = REFS[spec]
    # float64 reference rounded to the output dtype, as the reference's checks do
    check(got, np.asarray(fn(shaped(pairs, host))).astype(got.dtype), rtol, atol, spec)


@pytest.mark.gpu
@pytest.mark.parametrize("spec", IDS)
def test_kernels_meet_the_reference(spec):
    import torch
    from ptxc.package import ChainExecutor
    pairs = catalogue.build(spec)
    host = host_inputs(pairs)
    ex = ChainExecutor(Chain.from_kernels(pairs))
    ex.upload(host)
    ex.launch()
    torch.cuda.synchronize()
    got = ex.download()[final_output(pairs)].numpy()
    fn, rtol, atol = REFS[spec]
    check(got, np.asarray(fn(shaped(pairs, host))).astype(got.dtype), rtol, atol, spec)
