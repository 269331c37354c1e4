"""Machinery contract of the drop-in compiler (mirrors the reference's
``tests/test_machinery.py:277-332`` launch guards and ``:587-744`` loud
failures), restated on synthesised IR.

* a block collective (Sync / TreeHalve) under a partial block, a warp
  collective (WarpShuffle, warp Sync) under a partial warp: ``CompileError``;
* a warp collective whose active lanes fill whole warps passes the guards
  even though the block is partial;
* two KernelOps in one graph, a meta.json with no kernels or bytes that are
  not UTF-8, an unknown statement class, IR text that is not IR syntax, a
  structural field of the wrong type, a bad ``arch``: exit 1 from the CLI with
  ``compile.py:`` on stderr and no traceback, or ``CompileError`` in process.
"""

from __future__ import annotations

import dataclasses
import json
import subprocess
import sys

import pytest

from conftest import ROOT
from emmy_ir import synth
from emmy_ir.nodes import Dim
from emmy_ir.serialize import write_package
from ptxc import CompileError, Lowerer


def _cli(ir):
    return subprocess.run([sys.executable, str(ROOT / "compile.py"), str(ir)],
                          capture_output=True, text=True)


def _loud(r, needle):
    assert r.returncode == 1, r.stderr
    assert r.stdout == ""
    assert "compile.py:" in r.stderr and needle in r.stderr, r.stderr
    assert "Traceback" not in r.stderr


def _sum_kernel(lanes=256, strip=(), warp_sync=False):
    """A one-row block sum with 256 threads; ``lanes`` active lanes."""
    kop, meta = synth.reduce([1, 256], -1, "sum", block=256)
    tile = kop.body[0]
    body = tuple(s for s in tile.body if type(s).__name__ not in strip)
    if warp_sync:
        body = tuple(dataclasses.replace(s, warp=True) if type(s).__name__ == "Sync" else s
                     for s in body)
    axes = tuple(dataclasses.replace(a, extent=Dim(lanes)) if i == len(tile.axes) - 1 else a
                 for i, a in enumerate(tile.axes))
    tile = dataclasses.replace(tile, body=body, axes=axes)
    return dataclasses.replace(kop, body=(tile,)), meta


def test_partial_block_barrier_fails_loudly():
    kop, meta = _sum_kernel(lanes=200)
    with pytest.raises(CompileError, match="partial block"):
        Lowerer(kop, meta)


def test_full_warp_collective_passes_the_guards():
    # 128 active threads of a 256-thread block are four whole warps
    kop, meta = _sum_kernel(lanes=128, strip={"Sync", "TreeHalve"})
    Lowerer(kop, meta)


def test_partial_warp_shuffle_fails_loudly():
    kop, meta = _sum_kernel(lanes=100, strip={"Sync", "TreeHalve"})
    with pytest.raises(CompileError, match="partial warp"):
        Lowerer(kop, meta)


def test_partial_warp_sync_fails_loudly():
    kop, meta = _sum_kernel(lanes=100, strip={"TreeHalve", "WarpShuffle"}, warp_sync=True)
    with pytest.raises(CompileError, match="partial warp"):
        Lowerer(kop, meta)


@pytest.fixture
def package(tmp_path):
    kop, meta = synth.softmax([8, 256], entry="k_mach")
    return write_package(tmp_path / "pkg", kop, meta)


def test_multiple_kernel_ops_fail_loudly(package):
    doc = json.loads(package.read_text())
    name, node = next((k, v) for k, v in doc["nodes"].items() if v["op"] == "KernelOp")
    doc["nodes"][name + "_twin"] = node
    package.write_text(json.dumps(doc))
    _loud(_cli(package), "KernelOp")


def test_empty_meta_fails_loudly(package):
    (package.parent / "meta.json").write_text(json.dumps({"kernels": []}))
    _loud(_cli(package), "no kernels")


def test_invalid_utf8_meta_fails_loudly(package):
    (package.parent / "meta.json").write_bytes(b'{"kernels": ["\xff\xfe"]}')
    _loud(_cli(package), "cannot read")


def _edit_body(package, fn):
    doc = json.loads(package.read_text())
    node = next(v for v in doc["nodes"].values() if v["op"] == "KernelOp")
    node["op_fields"]["body"] = [fn(s) for s in node["op_fields"]["body"]]
    package.write_text(json.dumps(doc))


def test_unknown_statement_name_in_ir_fails_loudly(package):
    _edit_body(package, lambda s: s.replace("Tile(", "Tiled(", 1))
    _loud(_cli(package), "invalid IR")


def test_invalid_ir_syntax_fails_loudly(package):
    _edit_body(package, lambda s: s[: len(s) // 2])
    _loud(_cli(package), "invalid IR")


def test_malformed_structural_field_fails_loudly():
    kop, meta = synth.softmax([8, 256])
    tile = dataclasses.replace(kop.body[0], axes=5)          # not a tuple of Axis
    with pytest.raises(CompileError, match="invalid IR"):
        Lowerer(dataclasses.replace(kop, body=(tile,)), meta)


def test_bad_arch_fails_loudly():
    kop, meta = synth.softmax([8, 256])
    with pytest.raises(CompileError, match="arch"):
        Lowerer(kop, dict(meta, arch="gfx90a"))
