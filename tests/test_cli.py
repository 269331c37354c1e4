"""CLI contract of ``compile.py`` (mirrors the reference's ``tests/test_cli.py``).

Usage errors exit 2; a missing file, malformed JSON, a missing or malformed
meta.json, a non-ASCII entry or an unmatched IR exit 1 with ``compile.py:`` on
stderr, no traceback and an empty stdout; a valid IR exits 0 with the launch
plan on stdout.
"""

from __future__ import annotations

import json
import subprocess
import sys
import tempfile
from pathlib import Path

import pytest

from conftest import ROOT
from emmy_ir import synth
from emmy_ir.serialize import write_package


def run(*args, cwd=None, env=None):
    return subprocess.run([sys.executable, str(ROOT / "compile.py"), *args],
                          capture_output=True, text=True, cwd=cwd, env=env)


@pytest.fixture
def package(tmp_path):
    kop, meta = synth.rmsnorm(16, 256, eps=1e-5, entry="k_rms_cli")
    ir = write_package(tmp_path / "pkg", kop, meta)
    return ir


def test_no_argument_is_a_usage_error():
    r = run()
    assert r.returncode == 2
    assert "usage:" in r.stdout + r.stderr


def test_missing_file_fails_without_a_traceback():
    r = run(str(ROOT / "tests/does_not_exist.ir.json"))
    assert r.returncode == 1
    assert "compile.py:" in r.stderr
    assert "Traceback" not in r.stderr


def test_malformed_json_fails_loudly(tmp_path):
    path = tmp_path / "bad.ir.json"
    path.write_text("{not json")
    r = run(str(path))
    assert r.returncode == 1 and "compile.py:" in r.stderr and "Traceback" not in r.stderr


def test_valid_package_prints_the_plan(package):
    r = run(str(package))
    assert r.returncode == 0, r.stderr
    plan = json.loads(r.stdout)
    meta = json.loads((package.parent / "meta.json").read_text())["kernels"][0]
    assert plan["entry"] == meta["entry"]
    assert plan["arg_order"] == meta["arg_order"]
    assert plan["family"] == "rownorm" and plan["symbol"] == "emmy_rownorm_f32"
    assert r.stdout.isascii()


def test_missing_meta_fails_loudly(package, tmp_path):
    path = tmp_path / "k.ir.json"
    path.write_text(package.read_text())
    r = run(str(path))
    assert r.returncode == 1
    assert "meta.json" in r.stderr and "Traceback" not in r.stderr and r.stdout == ""


def _broken(package, tmp_path, mutate):
    meta = json.loads((package.parent / "meta.json").read_text())
    root = tmp_path / "broken"
    root.mkdir(exist_ok=True)
    (root / "k.ir.json").write_text(package.read_text())
    broken = json.loads(json.dumps(meta))
    mutate(broken)
    (root / "meta.json").write_text(json.dumps(broken))
    return run(str(root / "k.ir.json"))


@pytest.mark.parametrize("mutate,needle", [
    (lambda m: m["kernels"][0]["args"][0].pop("shape"), "shape"),
    (lambda m: m["kernels"][0]["args"][0].pop("dtype"), "dtype"),
    (lambda m: m["kernels"][0].__setitem__("arg_order", []), "arg_order"),
    (lambda m: m["kernels"][0].__setitem__("grid", [1, 1, 1, 1]), "3 integers"),
    (lambda m: m["kernels"][0].__setitem__("block", [256, 1]), "3 integers"),
    (lambda m: m["kernels"][0]["args"][0].__setitem__("scalar", "false"), "scalar"),
    (lambda m: m["kernels"][0].__setitem__("entry", "k_wrong"), "no kernel named"),
    (lambda m: m["kernels"][0].__setitem__("arch", "gfx90a"), "arch"),
    (lambda m: m["kernels"][0]["args"][2].__setitem__("dtype", "f128"), "dtype"),
    (lambda m: m["kernels"][0].__setitem__("grid", [0, 1, 1]), "positive"),
    (lambda m: m["kernels"][0].__setitem__("smem_bytes", -1), "smem_bytes"),
])
def test_strict_argument_and_launch_fields(package, tmp_path, mutate, needle):
    r = _broken(package, tmp_path, mutate)
    assert r.returncode == 1
    assert needle in r.stderr
    assert "Traceback" not in r.stderr
    assert r.stdout == ""


@pytest.mark.parametrize("field", ["grid", "block", "arg_order", "args"])
def test_missing_launch_field_fails_loudly(package, tmp_path, field):
    r = _broken(package, tmp_path, lambda m: m["kernels"][0].pop(field, None))
    assert r.returncode == 1 and field in r.stderr and "Traceback" not in r.stderr
    assert r.stdout == ""


def test_non_ascii_entry_fails_loudly(package, tmp_path):
    meta = json.loads((package.parent / "meta.json").read_text())
    ir = json.loads(package.read_text())
    for node in ir["nodes"].values():
        if node.get("op") == "KernelOp":
            node["op_fields"]["name"] = "k_café"
    meta["kernels"][0]["entry"] = "k_café"
    root = tmp_path / "na"
    root.mkdir()
    (root / "k.ir.json").write_text(json.dumps(ir))
    (root / "meta.json").write_text(json.dumps(meta))
    r = run(str(root / "k.ir.json"))
    assert r.returncode == 1 and "ASCII" in r.stderr and "Traceback" not in r.stderr
    assert r.stdout == ""


def test_deep_meta_fails_loudly(package, tmp_path):
    root = tmp_path / "deep"
    root.mkdir()
    (root / "k.ir.json").write_text(package.read_text())
    (root / "meta.json").write_text("[" * 20000 + "]" * 20000)
    r = run(str(root / "k.ir.json"))
    assert r.returncode == 1 and "meta.json" in r.stderr and "Traceback" not in r.stderr
    assert r.stdout == ""


def test_unmatched_ir_fails_loudly_without_fallback(package, tmp_path):
    ir = json.loads(package.read_text())
    for node in ir["nodes"].values():
        if node.get("op") == "KernelOp":
            # turn the squared-sum fold into a plain sum: no family computes
            # x * recip(sqrt(eps + sum(x) / n)) * w
            node["op_fields"]["body"] = [s.replace("args=('in2', 'in2')", "args=('in2', 'one_')")
                                         .replace("StridedLoop(axis=Axis(name='a1'", "StridedLoop(axis=Axis(name='a1'", 1)
                                         for s in node["op_fields"]["body"]]
    root = tmp_path / "um"
    root.mkdir()
    (root / "k.ir.json").write_text(json.dumps(ir))
    (root / "meta.json").write_text((package.parent / "meta.json").read_text())
    r = run(str(root / "k.ir.json"))
    assert r.returncode == 1
    assert "no B200 kernel family matches" in r.stderr
    assert r.stdout == ""


def test_invalid_ir_statement_is_a_compile_error(package, tmp_path):
    ir = json.loads(package.read_text())
    for node in ir["nodes"].values():
        if node.get("op") == "KernelOp":
            node["op_fields"]["body"] = ["Frobnicate(x=1)"]
    root = tmp_path / "inv"
    root.mkdir()
    (root / "k.ir.json").write_text(json.dumps(ir))
    (root / "meta.json").write_text((package.parent / "meta.json").read_text())
    r = run(str(root / "k.ir.json"))
    assert r.returncode == 1 and "invalid IR" in r.stderr and "Traceback" not in r.stderr


def test_integer_program_prints_its_plan_and_refusals_exit_1(tmp_path):
    """An integer pointwise package compiles to the pointwise_int plan; an
    integer op the reference cannot lower exits 1 with its message."""
    kop, meta = synth.pointwise(1000, ("maximum", ("subtract", "x0", "x1"), ("imm", 0)), "u8",
                                entry="k_int_cli")
    r = run(str(write_package(tmp_path / "ok", kop, meta)))
    assert r.returncode == 0, r.stderr
    plan = json.loads(r.stdout)
    assert plan["family"] == "pointwise_int" and plan["symbol"] == "emmy_pointwise_int"
    assert plan["pointwise"]["immediates"] == [0] and plan["pointwise"]["out_dtype"] == "u8"
    kop, meta = synth.pointwise(1000, ("negative", "x0"), "i32", entry="k_int_neg")
    r = run(str(write_package(tmp_path / "neg", kop, meta)))
    assert r.returncode == 1 and r.stdout == ""
    assert "unsupported integer op 'negative'" in r.stderr and "Traceback" not in r.stderr
