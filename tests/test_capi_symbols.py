"""The C-ABI library loads without a GPU and exports every symbol the header declares."""

from __future__ import annotations

import ctypes
import re

import pytest

from conftest import PKG, ROOT

HEADER = ROOT / "include" / "emmy_b200.h"


def declared_symbols():
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(emmy_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    path = PKG / "libemmyb200.so"
    if not path.exists():
        import importlib.util
        spec = importlib.util.spec_from_file_location("emmy_build", PKG / "build.py")
        mod = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(mod)
        mod.build()
    return ctypes.CDLL(str(path))


def test_header_declares_the_families():
    syms = declared_symbols()
    for s in ("emmy_reduce_f32", "emmy_rownorm_f32", "emmy_softmax_f32", "emmy_matvec_f64",
              "emmy_last_error", "emmy_get_device_status", "emmy_zero", "emmy_version"):
        assert s in syms


def test_library_exports_every_declared_symbol(lib):
    missing = [s for s in declared_symbols() if not hasattr(lib, s)]
    assert not missing, missing


def test_version_and_error_text_need_no_gpu(lib):
    assert lib.emmy_version() >= 100
    lib.emmy_last_error.restype = ctypes.c_char_p
    assert lib.emmy_last_error() is not None


def test_host_side_argument_checks_run_before_any_cuda_call(lib):
    # invalid sizes are rejected on the host with EMMY_ERR_INVALID (no device touched)
    lib.emmy_softmax_f32.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64,
                                     ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p]
    assert lib.emmy_softmax_f32(None, None, -1, 4, 1, None) == 1
    lib.emmy_last_error.restype = ctypes.c_char_p
    assert b"bad view" in lib.emmy_last_error()
    lib.emmy_rownorm_f32.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_int64] * 2 + \
        [ctypes.c_void_p] * 2 + [ctypes.c_int, ctypes.c_void_p]
    assert lib.emmy_rownorm_f32(None, None, None, None, 4, 4, None, None, 0, None) == 1
    assert lib.emmy_rownorm_f32(None, None, None, None, 0, 4, None, None, 0, None) == 0


def test_peer_slot_size_checked_on_the_host(lib):
    # a slot buffer smaller than world x rows_per_rank x N is refused before any launch
    lib.emmy_gemm_f32_rows_to_peers.argtypes = (
        [ctypes.c_void_p] * 4 + [ctypes.c_int64, ctypes.c_int, ctypes.c_int] +
        [ctypes.c_int64] * 4 + [ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64,
                                ctypes.c_void_p])
    lib.emmy_last_error.restype = ctypes.c_char_p
    rows = (ctypes.c_void_p * 8)(*([ctypes.c_void_p(256)] * 8))
    rc = lib.emmy_gemm_f32_rows_to_peers(ctypes.c_void_p(256), ctypes.c_void_p(256), None, rows,
                                         2 * 128 * 64 - 1, 2, 0, 128, 256, 64, 1024, 1,
                                         ctypes.c_void_p(256), ctypes.c_void_p(256), 64, None)
    assert rc == 1
    assert b"slot buffers" in lib.emmy_last_error()


def test_pointwise_program_checks_need_no_gpu(lib):
    vp, i32, i64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64
    lib.emmy_pointwise.argtypes = [vp, vp, i32, vp, vp, i32, vp, i32, vp, i32, i32, i32, vp, i32,
                                   i64, vp]
    lib.emmy_last_error.restype = ctypes.c_char_p
    ins = (vp * 1)(vp(16))
    dts = (i32 * 1)(0)
    # empty output: nothing to do, success without touching a device
    prog = (i32 * 5)(1, 1, 0, 0, 0)
    assert lib.emmy_pointwise(ins, dts, 1, None, None, 0, None, 0, prog, 1, 1, 0, vp(16), 0, 0,
                              None) == 0
    # unknown opcode, a step that overwrites an input register, a bad result register
    bad = (i32 * 5)(99, 1, 0, 0, 0)
    assert lib.emmy_pointwise(ins, dts, 1, None, None, 0, None, 0, bad, 1, 1, 0, vp(16), 0, 8,
                              None) == 1
    assert b"unknown opcode" in lib.emmy_last_error()
    clobber = (i32 * 5)(1, 0, 0, 0, 0)
    assert lib.emmy_pointwise(ins, dts, 1, None, None, 0, None, 0, clobber, 1, 1, 0, vp(16), 0, 8,
                              None) == 1
    assert lib.emmy_pointwise(ins, dts, 1, None, None, 0, None, 0, prog, 1, 7, 0, vp(16), 0, 8,
                              None) == 1
    assert b"result register" in lib.emmy_last_error()


def test_pointwise_broadcast_bounds_checked_on_the_host(lib):
    vp, i32, i64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64
    lib.emmy_pointwise_indexed.argtypes = [vp, vp, vp, i32, vp, vp, i32, vp, i32, vp, i32, i32, i32,
                                           vp, i32, i64, i64, vp]
    lib.emmy_last_error.restype = ctypes.c_char_p
    ins = (vp * 2)(vp(16), vp(32))
    dts = (i32 * 2)(0, 0)
    prog = (i32 * 5)(1, 2, 0, 1, 0)
    # input 1 read at (first + e) % 128 but holding only 100 elements
    idx = (i64 * 6)(0, 0, 0, 1, 128, 100)
    assert lib.emmy_pointwise_indexed(ins, dts, idx, 2, None, None, 0, None, 0, prog, 1, 2, 0,
                                      vp(64), 0, 0, 4096, None) == 1
    assert b"read past" in lib.emmy_last_error()
    # (first + e) / 32 for e < 4096 from first 1024 reaches element 159 of 128
    idx = (i64 * 6)(0, 0, 0, 32, 0, 128)
    assert lib.emmy_pointwise_indexed(ins, dts, idx, 2, None, None, 0, None, 0, prog, 1, 2, 0,
                                      vp(64), 0, 1024, 4096, None) == 1
    # a negative divisor
    idx = (i64 * 6)(0, 0, 0, -3, 0, 128)
    assert lib.emmy_pointwise_indexed(ins, dts, idx, 2, None, None, 0, None, 0, prog, 1, 2, 0,
                                      vp(64), 0, 0, 4096, None) == 1
    assert b"bad index" in lib.emmy_last_error()


def test_gemm_epilogue_bits_checked_on_the_host(lib):
    vp, i32, i64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64
    lib.emmy_gemm_f16.argtypes = [vp, vp, vp, vp, i64, i64, i64, i64, i32, i32, i32, vp]
    lib.emmy_gemm_f32.argtypes = [vp, vp, vp, vp, i64, i64, i64, i64, i64, i64, i64, i32, i32,
                                  i32, vp]
    lib.emmy_last_error.restype = ctypes.c_char_p
    assert lib.emmy_gemm_f16(vp(16), vp(16), None, vp(16), 1, 64, 64, 64, 1, 8, 0, None) == 1
    assert b"epilogue" in lib.emmy_last_error()
    # rounding to f16 first is an f16-matmul step only
    assert lib.emmy_gemm_f32(vp(16), vp(16), None, vp(16), 1, 64, 64, 64, 0, 0, 0, 1, 0, 4,
                             None) == 1
    assert b"epilogue" in lib.emmy_last_error()


def test_launcher_refuses_to_run_without_the_library(tmp_path, monkeypatch):
    import ptxc.launch as L
    monkeypatch.setattr(L, "_LIB", None)
    monkeypatch.setenv("EMMY_B200_LIB", str(tmp_path / "missing.so"))
    with pytest.raises(L.LibraryError):
        L.load_library()
