"""GPU parity of the attention family.

IR cases are synthesised in the ``w_a_head64`` statement shape: the f32
fixture shapes (q [S,D], kt [D,S] pre-transposed, v [S,Dv]) on CUDA cores,
and the f16 benchmark shapes (q, k, v [B,H,S,D]) on the tcgen05 kernel.

Tolerance per output element, against the float64 oracle
``oracle.formulas.attention_bhsd`` (``tests/parity.py``): each output is a
convex combination of values, so its error is bounded relative to the row's
own scale ``sum_j p_j |v_j|`` (float64): f32 ``|d| <= 1e-5 * sum_j p_j|v_j|``;
f16 operands with f32 softmax and accumulation ``|d| <= 1e-3 * sum_j p_j|v_j|
+ u * |ref|`` with ``u = 2^-11`` (one rounding) for an f16 output.
"""

from __future__ import annotations

import numpy as np
import pytest

from emmy_ir import synth
from gpu_util import run_on_gpu, shaped
from oracle import formulas as F
from oracle.interp import run_ir
from parity import check

pytestmark = pytest.mark.gpu


def _ref(meta, host, kt):
    x = shaped(meta, host)
    k = np.swapaxes(x["k"], -1, -2) if kt else x["k"]
    div = [a["data"][0] for a in meta["args"] if a["name"] == "div_c1"][0]
    ref = F.attention_bhsd(x["q"], k, x["v"], 1.0 / div, out_dtype=np.float64)
    return x, ref, F.attention_abs_scale(x["q"], k, x["v"], 1.0 / div)


F32_CASES = [
    ("v_a_128", dict(B=1, H=1, S=128, D=128, k_transposed=True, scale_div=11.313708)),
    ("v_a_32x256", dict(B=1, H=1, S=32, D=256, Dv=32, k_transposed=True, scale_div=16.0)),
    ("v_a_64x128", dict(B=1, H=1, S=64, D=128, Dv=64, k_transposed=True, scale_div=8.0)),
    ("w_a_256", dict(B=1, H=1, S=256, D=64, k_transposed=True, scale_div=8.0)),
    ("w_a_head64", dict(B=1, H=1, S=128, D=64, k_transposed=True, scale_div=8.0)),
    ("bhsd_2x3x100x48", dict(B=2, H=3, S=100, D=48, Dv=16)),
]


@pytest.mark.parametrize("name,kw", F32_CASES, ids=[c[0] for c in F32_CASES])
def test_attention_f32(name, kw):
    kop, meta = synth.attention(dtype="f32", **kw)
    plan, host, out = run_on_gpu(kop, meta)
    assert plan["family"] == "attention_f32"
    x, ref, scale = _ref(meta, host, kw.get("k_transposed", False))
    got = out["o"].reshape(ref.shape).astype(np.float64)
    check(got, ref, scale, case=f"attention_f32 {name}", family="attention", dtype="f32")
    if kw["S"] * kw["D"] <= 64 * 128:
        # the interpreter is itself an f32 evaluation: the two differ by at
        # most the sum of their errors
        interp = run_ir(kop, meta, host)["o"].reshape(ref.shape).astype(np.float64)
        check(got, interp, scale, case=f"attention_f32 {name} vs interpreter",
              family="attention", dtype="f32", rtol=2e-5)


F16_CASES = [
    ("K5_8x32x512x128_f16out", dict(B=8, H=32, S=512, D=128, out_dtype="f16")),
    ("K5_2x4x512x128_f32out", dict(B=2, H=4, S=512, D=128, out_dtype="f32")),
] + [
    (f"sweep_S{S}_D{D}", dict(B=2, H=4, S=S, D=D, out_dtype="f16"))
    for D in (16, 32, 64, 96, 256) for S in (16, 128, 512)
] + [
    # head dims run by the next-wider tensor-core kernel (TMA zero-fills the
    # columns past d): multiples of 8 that are not multiples of 16, d between
    # the widths, f32 output, ragged key counts
    ("d24_S130_f32out", dict(B=2, H=3, S=130, D=24, out_dtype="f32")),
    ("d48_S200", dict(B=1, H=5, S=200, D=48, out_dtype="f16")),
    ("d96_S512_f32out", dict(B=2, H=4, S=512, D=96, out_dtype="f32")),
    ("d104_S77", dict(B=3, H=2, S=77, D=104, out_dtype="f16")),
    ("d200_S256", dict(B=1, H=4, S=256, D=200, out_dtype="f16")),
    ("d16_tiles_x600", dict(B=6, H=100, S=256, D=16, out_dtype="f16")),

    ("ragged_S200_D64", dict(B=1, H=3, S=200, D=64, out_dtype="f32")),
    # more query tiles than resident CTAs: each persistent CTA walks several
    ("tiles_S200_D64_x1200", dict(B=6, H=100, S=200, D=64, out_dtype="f32")),
    ("tiles_S512_D256_x320", dict(B=2, H=40, S=512, D=256, out_dtype="f16")),
    # D = 128, ragged: a last key block with a single valid key, one partial
    # block, and ragged tiles over several passes of the persistent CTAs
    ("ragged_S129_D128", dict(B=1, H=3, S=129, D=128, out_dtype="f32")),
    ("ragged_S65_D128", dict(B=2, H=2, S=65, D=128, out_dtype="f16")),
    ("ragged_S200_D128_x600", dict(B=3, H=100, S=200, D=128, out_dtype="f16")),
    ("ragged_S200_D256", dict(B=1, H=3, S=200, D=256, out_dtype="f32")),
    ("ragged_S130_D256_x300", dict(B=3, H=50, S=130, D=256, out_dtype="f16")),
    ("kt_f16_fallback", dict(B=1, H=2, S=64, D=32, out_dtype="f32", k_transposed=True)),
]


@pytest.mark.parametrize("name,kw", F16_CASES, ids=[c[0] for c in F16_CASES])
def test_attention_f16(name, kw):
    kop, meta = synth.attention(dtype="f16", **kw)
    plan, host, out = run_on_gpu(kop, meta)
    assert plan["family"] == "attention_f16"
    x, ref, scale = _ref(meta, host, kw.get("k_transposed", False))
    got = out["o"].reshape(ref.shape).astype(np.float64)
    check(got, ref, scale, case=f"attention_f16 {name}", family="attention", dtype="f16",
          out_dtype=kw["out_dtype"])
