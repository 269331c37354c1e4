"""The same IR gives a byte-identical launch plan across runs, working
directories and hash seeds (the reference's ``tests/test_determinism.py``
property, applied to the plan)."""

from __future__ import annotations

import os
import subprocess
import sys

import pytest

from conftest import ROOT
from emmy_ir import synth
from emmy_ir.serialize import write_package


@pytest.fixture(scope="module")
def ir_path(tmp_path_factory):
    kop, meta = synth.softmax([4, 8, 256], entry="k_det")
    return write_package(tmp_path_factory.mktemp("det"), kop, meta)


def compile_once(ir, cwd, hashseed):
    env = dict(os.environ)
    env["PYTHONHASHSEED"] = str(hashseed)
    r = subprocess.run([sys.executable, str(ROOT / "compile.py"), str(ir)],
                       capture_output=True, text=True, cwd=cwd, env=env)
    assert r.returncode == 0, r.stderr
    return r.stdout


def test_two_runs_are_identical(ir_path):
    assert compile_once(ir_path, ROOT, 0) == compile_once(ir_path, ROOT, 0)


def test_working_directory_does_not_change_the_output(ir_path):
    assert compile_once(ir_path, ROOT, 1) == compile_once(ir_path, "/tmp", 1)


def test_hash_seed_does_not_change_the_output(ir_path):
    assert compile_once(ir_path, ROOT, 2) == compile_once(ir_path, ROOT, 3)
