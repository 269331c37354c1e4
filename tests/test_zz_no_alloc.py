"""The no-allocation long-row reduction (``emmy_reduce_f32_noalloc``).

Callers that cannot allocate device memory at call time (a memory pool fixed at
start-up and owned by the host program, allocator callbacks that must not
re-enter the allocator, loops that cannot afford an allocation's implicit
synchronisation) use this entry point: its per-CTA
partials live in a fixed array inside the library instead of a workspace the
caller passes.  This test calls it through the C ABI and checks it against the
workspace entry point (``emmy_reduce_f32``) on the same input, within the
reduction tolerance the other GPU tests use (``|d| <= 1e-5 * sum|x|``), on two
calls in a row (the second on a shorter row, so stale partials from the first
call are present in the shared array).  Collected last so that a run stopping
at the first failure has already run every other test.
"""

from __future__ import annotations

import ctypes

import pytest

pytestmark = pytest.mark.gpu

RTOL = 1e-5


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def test_noalloc_reduction_matches_the_workspace_entry_point_twice():
    import torch
    from ptxc.launch import load_library
    lib = load_library()
    g = torch.Generator(device="cuda").manual_seed(1234)
    for call, (n, op, pre, mean) in enumerate([(9_000_001, 0, 0, False), (3_000_017, 0, 1, True)]):
        x = torch.randn(n, device="cuda", generator=g)
        count = torch.tensor([float(n)], device="cuda") if mean else None
        ws_bytes = int(lib.emmy_reduce_workspace_bytes(1, n, 1))
        ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device="cuda")
        y_ref = torch.full((1,), float("nan"), device="cuda")
        rc = lib.emmy_reduce_f32(_p(x), _p(y_ref), 1, n, 1, op, pre,
                                 _p(count) if mean else None, _p(ws), ws_bytes, None)
        assert rc == 0, lib.emmy_last_error()
        y = torch.full((1,), float("nan"), device="cuda")
        rc = lib.emmy_reduce_f32_noalloc(_p(x), _p(y), n, op, pre,
                                         _p(count) if mean else None, None)
        assert rc == 0, lib.emmy_last_error()
        torch.cuda.synchronize()
        scale = (x.double() ** 2).sum() if pre == 1 else x.double().abs().sum()
        if mean:
            scale = scale / n
        assert abs(float(y) - float(y_ref)) <= RTOL * float(scale), (call, float(y), float(y_ref))


def test_noalloc_rejects_rows_beyond_its_scratch():
    from ptxc.launch import load_library
    lib = load_library()
    rc = lib.emmy_reduce_f32_noalloc(ctypes.c_void_p(16), ctypes.c_void_p(16), 4096 * 16384 + 1,
                                     0, 0, None, None)
    assert rc == 1
    assert b"limit" in lib.emmy_last_error()
