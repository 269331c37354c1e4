"""GPU parity of the tcgen05 f16 GEMM family (f32 accumulation, bias + ReLU, BMM).

IR cases: the K3a benchmark (4096x2048 @ 2048x8192 + bias, ReLU; f16 and f32
output) and K3b (BMM 64 x 512^3), plus edge tiles; direct C-ABI cases cover
shapes that take the CUDA-core fallback (K or N not a multiple of 8).

Tolerance per output element (f16 inputs, f32 accumulation, north-star
1e-3): ``|got - ref| <= 1e-3 * (|A| @ |B| + |bias|) + u * |ref|`` with
``u = 2^-11`` (one f16 rounding) for f16 output and 0 for f32 output.
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

RTOL = 1e-3
STD = 2048 ** -0.5

IR_CASES = [
    ("K3a_bias_relu_f16out", dict(M=4096, N=8192, K=2048, dtype="f16", out_dtype="f16", bias=True,
                                  relu=True, tm=128, tn=128, rm=8, rn=8,
                                  a_init={"dist": "normal", "std": STD},
                                  b_init={"dist": "normal", "std": STD},
                                  bias_init={"dist": "normal", "std": 0.02})),
    ("K3a_bias_relu_f32out", dict(M=4096, N=8192, K=2048, dtype="f16", out_dtype="f32", bias=True,
                                  relu=True, tm=128, tn=128, rm=8, rn=8,
                                  a_init={"dist": "normal", "std": STD},
                                  b_init={"dist": "normal", "std": STD},
                                  bias_init={"dist": "normal", "std": 0.02})),
    ("K3b_bmm_64x512", dict(M=512, N=512, K=512, batch=64, dtype="f16", out_dtype="f16",
                            tm=128, tn=128, rm=8, rn=8,
                            a_init={"dist": "normal", "std": STD}, b_init={"dist": "normal", "std": STD})),
    ("edge_tiles_192x136x72", dict(M=192, N=136, K=72, dtype="f16", out_dtype="f32", bias=True,
                                   tm=64, tn=8, rm=4, rn=1, bk=8)),
    ("one_tile_128x256x64", dict(M=128, N=256, K=64, dtype="f16", out_dtype="f16", tm=64, tn=64)),
    # CTA-pair kernel with a partial last round of tiles: 80 tiles on 74
    # clusters with bias + ReLU, and the K3b shape with f32 output
    ("pair_tail_split_40x256x512x256", dict(M=256, N=512, K=256, batch=40, dtype="f16",
                                            out_dtype="f32", bias=True, relu=True, tm=128,
                                            tn=128, rm=8, rn=8,
                                            a_init={"dist": "normal", "std": STD},
                                            b_init={"dist": "normal", "std": STD})),
    ("pair_tail_split_K3b_f32out", dict(M=512, N=512, K=512, batch=64, dtype="f16",
                                        out_dtype="f32", tm=128, tn=128, rm=8, rn=8,
                                        a_init={"dist": "normal", "std": STD},
                                        b_init={"dist": "normal", "std": STD})),
    # 256 x 512 pair tiles (chosen: 144 of them take as many rounds as 288 of
    # 256 x 256): ragged in M (520), N (1000: the second half of the last
    # tile partial) and K (136), with bias + ReLU, f16 and f32 output
    ("wide_pair_tiles_ragged_24x520x1000x136", dict(M=520, N=1000, K=136, batch=24, dtype="f16",
                                                    out_dtype="f16", bias=True, relu=True, tm=8,
                                                    tn=8, rm=1, rn=1, bk=8,
                                                    a_init={"dist": "normal", "std": STD},
                                                    b_init={"dist": "normal", "std": STD})),
    ("wide_pair_tiles_ragged_f32out", dict(M=520, N=1000, K=136, batch=24, dtype="f16",
                                           out_dtype="f32", bias=True, tm=8, tn=8, rm=1, rn=1,
                                           bk=8, a_init={"dist": "normal", "std": STD},
                                           b_init={"dist": "normal", "std": STD})),
]


def _check(x, got, bias=None, relu=False, f16_out=True, case="gemm_f16"):
    ref = F.matmul(x["A"], x["B"], bias, relu, out_dtype=np.float64)
    scale = F.matmul_abs_bound(x["A"], x["B"], bias)
    check(got.reshape(ref.shape), ref, scale, case=case, family="gemm_f16", dtype="f16",
          out_dtype="f16" if f16_out else "f32")


@pytest.mark.parametrize("name,kw", IR_CASES, ids=[c[0] for c in IR_CASES])
def test_gemm_f16_ir(name, kw):
    kop, meta = synth.matmul(**kw)
    plan, host, out = run_on_gpu(kop, meta)
    assert plan["family"] == "gemm_f16"
    x = shaped(meta, host)
    _check(x, out["C"], x.get("bias"), kw.get("relu", False), kw["out_dtype"] == "f16",
           case=f"gemm_f16 {name}")


@pytest.mark.parametrize("M,N,K,batch,out", [(33, 30, 17, 1, 1), (5, 7, 9, 2, 0), (64, 24, 40, 1, 1),
                                             (300, 200, 100, 1, 0)])
def test_gemm_f16_cabi_fallback_and_edges(M, N, K, batch, out):
    import torch
    from ptxc.launch import load_library
    lib = load_library()
    g = torch.Generator(device="cuda").manual_seed(M + N + K)
    A = torch.randn(batch, M, K, device="cuda", generator=g).half()
    B = torch.randn(batch, K, N, device="cuda", generator=g).half()
    C = torch.full((batch, M, N), float("nan"), device="cuda",
                   dtype=torch.float16 if out else torch.float32)
    P = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    rc = lib.emmy_gemm_f16(P(A), P(B), None, P(C), batch, M, N, K, out, 0, 0, None)
    assert rc == 0, lib.emmy_last_error()
    torch.cuda.synchronize()
    ref = torch.bmm(A.double(), B.double())
    scale = torch.bmm(A.abs().double(), B.abs().double())
    u = 2.0 ** -11 if out else 0.0
    assert torch.all((C.double() - ref).abs() <= RTOL * scale + u * ref.abs())
