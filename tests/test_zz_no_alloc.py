"""The no-allocation long-row reduction (``emmy_reduce_f32_noalloc``).

Callers that cannot allocate device memory at call time (a memory pool fixed at
start-up and owned by the host program, allocator callbacks that must not
re-enter the allocator, loops that cannot afford an allocation's implicit
synchronisation) use this entry point: its per-CTA partials live in a fixed
array inside the library instead of a workspace the caller passes.

Each case calls it through the C ABI twice in a row (the second call on a
shorter row, so stale partials of the first call are present in the shared
array) and checks every result two ways, with the reduction tolerance the other
GPU tests use:

* against the workspace entry point (``emmy_reduce_f32``) on the same input:
  ``|d| <= 1e-5 * sum|pre(x)|`` for sums (the scale of the sum), exactly equal
  for max and min;
* against a float64 reduction of the same input: the same bounds.

One more case reduces a row of exactly the 67,108,864-element limit (every
partial slot and the finish kernel's full read), and rows beyond it are
rejected on the host.  Collected last so that a run stopping at the first
failure has already run every other test.
"""

from __future__ import annotations

import ctypes

import pytest

pytestmark = pytest.mark.gpu

RTOL = 1e-5
LIMIT = 4096 * 16384
OPS = {0: "sum", 1: "max", 2: "min"}
PRES = {0: "identity", 1: "square", 2: "abs"}


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def _f64_reference(x, op, pre, mean):
    v = x.double()
    if pre == 1:
        v = v * v
    elif pre == 2:
        v = v.abs()
    if op == 0:
        r = v.sum()
        scale = v.abs().sum()
        if mean:
            r, scale = r / x.numel(), scale / x.numel()
        return float(r), float(scale)
    return float(v.max() if op == 1 else v.min()), 0.0


def _both(lib, x, op, pre, mean):
    import torch
    n = x.numel()
    count = torch.tensor([float(n)], device="cuda") if mean else None
    ws_bytes = int(lib.emmy_reduce_workspace_bytes(1, n, 1))
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device="cuda")
    y_ws = torch.full((1,), float("nan"), device="cuda")
    rc = lib.emmy_reduce_f32(_p(x), _p(y_ws), 1, n, 1, op, pre, _p(count) if mean else None,
                             _p(ws), ws_bytes, None)
    assert rc == 0, lib.emmy_last_error()
    y = torch.full((1,), float("nan"), device="cuda")
    rc = lib.emmy_reduce_f32_noalloc(_p(x), _p(y), n, op, pre, _p(count) if mean else None, None)
    assert rc == 0, lib.emmy_last_error()
    torch.cuda.synchronize()
    return float(y), float(y_ws)


def _check(got, want, scale, op, what):
    if op == 0:
        assert abs(got - want) <= RTOL * scale, (what, got, want, scale)
    else:
        assert got == want, (what, got, want)


@pytest.mark.parametrize("pre", sorted(PRES), ids=[PRES[k] for k in sorted(PRES)])
@pytest.mark.parametrize("op", sorted(OPS), ids=[OPS[k] for k in sorted(OPS)])
def test_noalloc_matches_the_workspace_entry_point_and_float64_twice(op, pre):
    import torch
    from ptxc.launch import load_library
    lib = load_library()
    g = torch.Generator(device="cuda").manual_seed(1234 + 10 * op + pre)
    for call, (n, mean) in enumerate([(9_000_001, False), (3_000_017, op == 0)]):
        x = torch.randn(n, device="cuda", generator=g)
        got, ws = _both(lib, x, op, pre, mean)
        want, scale = _f64_reference(x, op, pre, mean)
        _check(got, ws, scale, op, f"call {call}: noalloc vs emmy_reduce_f32")
        _check(got, want if op == 0 else float(torch.tensor(want, dtype=torch.float32)), scale, op,
               f"call {call}: noalloc vs float64")


def test_noalloc_row_at_the_limit():
    """n = 4096 x 16384: all 4096 partial slots written and read by the finish step."""
    import torch
    from ptxc.launch import load_library
    lib = load_library()
    g = torch.Generator(device="cuda").manual_seed(99)
    x = torch.rand(LIMIT, device="cuda", generator=g) - 0.5
    x[-1] = 7.5                                   # the last element lands in the last slot
    for op in (0, 1):
        got, ws = _both(lib, x, op, 0, False)
        want, scale = _f64_reference(x, op, 0, False)
        _check(got, ws, scale, op, "limit: noalloc vs emmy_reduce_f32")
        _check(got, want, scale, op, "limit: noalloc vs float64")
    assert got == 7.5
    del x
    torch.cuda.empty_cache()


def test_noalloc_rejects_rows_beyond_its_scratch():
    from ptxc.launch import load_library
    lib = load_library()
    rc = lib.emmy_reduce_f32_noalloc(ctypes.c_void_p(16), ctypes.c_void_p(16), LIMIT + 1,
                                     0, 0, None, None)
    assert rc == 1
    assert b"limit" in lib.emmy_last_error()
