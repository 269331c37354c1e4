"""GPU parity of the f32 and f64 CUDA-core GEMM family (plain, batched, split-K, epilogue).

IR cases are the reference fixture shapes (``v_m_*``, ``w_m_*``), the K4a
benchmark (split-K 256x65536x256 in 64 partitions, U(-1,1) inputs) and an
epilogue case, compiled to plans and run through the C-ABI; direct C-ABI
cases cover shapes the TMA path cannot take (K or N not a multiple of 4).

Tolerance per output element: ``|got - ref| <= 1e-5 * (|A| @ |B|)`` (the
dot product's own scale, f64 reference), plus ``|bias|`` when a bias is added;
f64 operands (the reference's fma.rn.f64 accumulate): ``1e-13`` of the same
scale against an exact-as-possible reference (``math.fsum`` rows).
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

from emmy_ir import synth
from gpu_util import run_on_gpu, shaped
from oracle import formulas as F
from parity import check

pytestmark = pytest.mark.gpu

RTOL = 1e-5

IR_CASES = [
    ("v_m_256", dict(M=256, N=256, K=256)),
    ("v_m_rect_small_splitk16", dict(M=64, N=32, K=128, splits=16, tm=32, tn=32, rm=2, rn=2, bk=8)),
    ("v_m_tall_split2", dict(M=512, N=64, K=128, splits=2)),
    ("v_m_wide_split16", dict(M=128, N=512, K=64, splits=16, bk=4)),
    ("w_m_1024_split4", dict(M=1024, N=128, K=128, splits=4)),
    ("w_m_k96_split4", dict(M=128, N=64, K=96, splits=4, bk=8)),
    ("w_m_batch_split16", dict(M=64, N=64, K=64, batch=4, splits=16, bk=4)),
    ("K4a_splitk64", dict(M=256, N=256, K=65536, splits=64, tm=128, tn=128, rm=8, rn=8,
                          a_init={"dist": "uniform", "low": -1.0, "high": 1.0},
                          b_init={"dist": "uniform", "low": -1.0, "high": 1.0})),
    ("bias_relu_192x320x200", dict(M=192, N=320, K=200, bias=True, relu=True, tm=64, tn=64, bk=8)),
    ("batch3_bias", dict(M=128, N=64, K=48, batch=3, bias=True, bk=16)),
]


@pytest.mark.parametrize("name,kw", IR_CASES, ids=[c[0] for c in IR_CASES])
def test_gemm_f32_ir(name, kw):
    kop, meta = synth.matmul(**kw)
    plan, host, out = run_on_gpu(kop, meta)
    assert plan["family"] == "gemm_f32"
    x = shaped(meta, host)
    ref = F.matmul(x["A"], x["B"], x.get("bias"), kw.get("relu", False), out_dtype=np.float64)
    scale = F.matmul_abs_bound(x["A"], x["B"], x.get("bias"))
    got = out["C"].reshape(ref.shape).astype(np.float64)
    check(got, ref, scale, case=f"gemm_f32 {name}", family="gemm_f32", dtype="f32")


@pytest.mark.parametrize("M,N,K,batch", [(33, 30, 17, 1), (5, 7, 9, 2), (130, 4, 1024, 1),
                                         (1, 1, 1, 1), (129, 257, 64, 1)])
def test_gemm_f32_cabi_odd_shapes(M, N, K, batch):
    import torch
    from ptxc.launch import load_library
    lib = load_library()
    g = torch.Generator(device="cuda").manual_seed(M * 1000 + N)
    A = torch.randn(batch, M, K, device="cuda", generator=g)
    B = torch.randn(batch, K, N, device="cuda", generator=g)
    C = torch.full((batch, M, N), float("nan"), device="cuda")
    P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    rc = lib.emmy_gemm_f32(P(A), P(B), None, P(C), batch, M, N, K, M * K, K * N, M * N, 0, 0, 0, None)
    assert rc == 0, lib.emmy_last_error()
    torch.cuda.synchronize()
    ref = torch.bmm(A.double(), B.double())
    scale = torch.bmm(A.abs().double(), B.abs().double())
    assert torch.all((C.double() - ref).abs() <= RTOL * scale + 1e-30)


def test_gemm_f32_accumulate_adds_into_c():
    import torch
    from ptxc.launch import load_library
    lib = load_library()
    A = torch.randn(96, 64, device="cuda")
    B = torch.randn(64, 80, device="cuda")
    C0 = torch.randn(96, 80, device="cuda")
    C = C0.clone()
    P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    for splits in (1, 4):
        C.copy_(C0)
        assert lib.emmy_gemm_f32(P(A), P(B), None, P(C), 1, 96, 80, 64, 0, 0, 0, splits, 1, 0, None) == 0
        torch.cuda.synchronize()
        ref = C0.double() + A.double() @ B.double()
        scale = C0.double().abs() + A.abs().double() @ B.abs().double()
        assert torch.all((C.double() - ref).abs() <= RTOL * scale)


def test_gemm_f32_rejects_relu_on_partial_sums():
    from ptxc.launch import load_library
    lib = load_library()
    rc = lib.emmy_gemm_f32(ctypes.c_void_p(16), ctypes.c_void_p(16), None, ctypes.c_void_p(16),
                           1, 8, 8, 8, 0, 0, 0, 4, 0, 2, None)
    assert rc == 1


F64_CASES = [
    ("v_m_256_f64", dict(M=256, N=256, K=256)),
    ("tall_split2_f64", dict(M=512, N=64, K=128, splits=2)),
    ("batch4_split16_f64", dict(M=64, N=64, K=64, batch=4, splits=16, bk=4)),
    ("bias_relu_f64", dict(M=192, N=320, K=200, bias=True, relu=True, tm=64, tn=64, bk=8)),
    ("odd_k_f64", dict(M=96, N=80, K=50, tm=32, tn=16, rm=2, rn=2, bk=2)),
    ("splitk_f64_4096", dict(M=128, N=128, K=4096, splits=8, tm=128, tn=128, rm=8, rn=8, bk=16)),
]


def _exact_matmul(A, B):
    """float64 product with every dot product summed exactly (then rounded once)."""
    import math
    out = np.empty((A.shape[0], B.shape[1]))
    for i in range(A.shape[0]):
        prod = A[i][:, None] * B            # products: exact only to f64, like an fma chain
        out[i] = [math.fsum(prod[:, j]) for j in range(B.shape[1])]
    return out


@pytest.mark.parametrize("name,kw", F64_CASES, ids=[c[0] for c in F64_CASES])
def test_gemm_f64_ir(name, kw):
    kop, meta = synth.matmul(dtype="f64", **kw)
    plan, host, out = run_on_gpu(kop, meta)
    assert plan["family"] == "gemm_f64"
    x = shaped(meta, host)
    A, B = x["A"], x["B"]
    if A.ndim == 2:
        A, B = A[None], B[None]
    ref = np.stack([_exact_matmul(a, b) for a, b in zip(A, B)])
    scale = np.stack([np.abs(a) @ np.abs(b) for a, b in zip(A, B)])
    if "bias" in x:
        ref = ref + x["bias"]
        scale = scale + np.abs(x["bias"])
    if kw.get("relu"):
        ref = np.maximum(ref, 0)
    got = out["C"].reshape(ref.shape)
    check(got, ref, scale, case=f"gemm_f64 {name}", family="gemm_f64", dtype="f64", rtol=1e-13)


@pytest.mark.parametrize("M,N,K,batch", [(33, 30, 17, 1), (5, 7, 9, 2), (130, 4, 1024, 1),
                                         (1, 1, 1, 1), (129, 257, 64, 1)])
def test_gemm_f64_cabi_odd_shapes(M, N, K, batch):
    import torch
    from ptxc.launch import load_library
    lib = load_library()
    g = torch.Generator(device="cuda").manual_seed(M * 1000 + N)
    A = torch.randn(batch, M, K, device="cuda", generator=g, dtype=torch.float64)
    B = torch.randn(batch, K, N, device="cuda", generator=g, dtype=torch.float64)
    C = torch.full((batch, M, N), float("nan"), device="cuda", dtype=torch.float64)
    P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    rc = lib.emmy_gemm_f64(P(A), P(B), None, P(C), batch, M, N, K, M * K, K * N, M * N, 0, 0, 0, None)
    assert rc == 0, lib.emmy_last_error()
    torch.cuda.synchronize()
    ref = torch.bmm(A, B)
    scale = torch.bmm(A.abs(), B.abs())
    assert torch.all((C - ref).abs() <= 1e-13 * scale + 1e-300)


def test_gemm_f64_accumulate_adds_into_c():
    import torch
    from ptxc.launch import load_library
    lib = load_library()
    A = torch.randn(96, 64, device="cuda", dtype=torch.float64)
    B = torch.randn(64, 80, device="cuda", dtype=torch.float64)
    C0 = torch.randn(96, 80, device="cuda", dtype=torch.float64)
    C = C0.clone()
    P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    for splits in (1, 4):
        C.copy_(C0)
        assert lib.emmy_gemm_f64(P(A), P(B), None, P(C), 1, 96, 80, 64, 0, 0, 0, splits, 1, 0, None) == 0
        torch.cuda.synchronize()
        ref = C0 + A @ B
        scale = C0.abs() + A.abs() @ B.abs()
        assert torch.all((C - ref).abs() <= 1e-13 * scale)


@pytest.mark.parametrize("M,N,K,splits", [(200, 196, 4096, 0), (136, 260, 1000, 1),
                                          (256, 128, 8192, 8)])
def test_rows_to_peers_single_owner_matches_the_plain_gemm(M, N, K, splits):
    """The fused split-K kernel with one owner (this GPU): auto-widened or
    caller splits, a bias, ragged 128 x 128 tiles.  Its slot must equal the
    plain f32 GEMM within the GEMM tolerance, and the tile workspace and
    arrival counters must be left zero for the next call (checked over two
    calls)."""
    import torch
    from ptxc.launch import load_library
    lib = load_library()
    g = torch.Generator(device="cuda").manual_seed(M + N + K)
    A = torch.rand(M, K, device="cuda", generator=g) * 2 - 1
    B = torch.rand(K, N, device="cuda", generator=g) * 2 - 1
    bias = torch.randn(N, device="cuda", generator=g)
    P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    plain = torch.empty(M, N, device="cuda")
    assert lib.emmy_gemm_f32(P(A), P(B), P(bias), P(plain), 1, M, N, K, 0, 0, 0, splits, 0, 1,
                             None) == 0, lib.emmy_last_error()
    slots = torch.full((1, M, N), float("nan"), device="cuda")
    ws = torch.zeros(M * N, device="cuda")
    tiles = ((M + 63) // 64) * ((N + 63) // 64)
    counters = torch.zeros(tiles, dtype=torch.int32, device="cuda")
    rows = (ctypes.c_void_p * 8)(P(slots), *([ctypes.c_void_p(0)] * 7))
    for _ in range(2):
        slots.fill_(float("nan"))
        rc = lib.emmy_gemm_f32_rows_to_peers(P(A), P(B), P(bias), rows, slots.numel(), 1, 0, M,
                                             M, N, K, splits, P(ws), P(counters), tiles, None)
        assert rc == 0, lib.emmy_last_error()
        torch.cuda.synchronize()
        ref = A.double() @ B.double() + bias.double()
        scale = A.double().abs() @ B.double().abs() + bias.double().abs()
        got = slots[0].double()
        assert torch.all((got - ref).abs() <= RTOL * scale), "fused slot differs from float64"
        assert torch.all((got - plain.double()).abs() <= 2 * RTOL * scale), "fused vs plain GEMM"
        assert int(torch.count_nonzero(ws)) == 0, "tile workspace not left zero"
        assert int(torch.count_nonzero(counters)) == 0, "arrival counters not left zero"
