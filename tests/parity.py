"""Parity bounds at the north-star tolerances, and a log of the observed errors.

Every GPU parity check of a kernel family against the float64 oracle (or
against the reference's own PTX) goes through ``check``:

    |got - ref| <= rtol * scale + u * |ref| + floor          (per element)

* ``rtol``: 1e-5 for f32 arithmetic, 1e-3 for f16 operands with f32
  accumulation, 1e-12 for f64 -- the tolerances the north star states;
* ``u``: one rounding of the output type, 2^-11 for an f16 output (the
  result is rounded once at the store), else 0;
* ``floor``: the output type's resolution near zero -- half the f16 subnormal
  step (2^-25) for f16 outputs, 1e-30 for f32 (flushed denormals), 0 for f64;
* ``scale``: the magnitude each family's rounding error grows with, computed
  in float64 from the inputs (``oracle.formulas``):
    - softmax, rms / l2 norm (products and positive sums, no cancellation):
      ``|ref|`` itself, i.e. a plain relative bound;
    - layer norm: ``(|x| + |mean|) * rstd * |gamma| + |beta|``;
    - sums and means: the sum (mean) of ``|pre(x)|``;
    - matmul, matvec, dot: ``|A| @ |B| (+ |bias|)``;
    - attention: ``sum_j p_j |v_j|``, the row's own convex-combination scale.

With ``EMMY_PARITY_LOG`` set to a file path, each check appends one JSON line:
the case, family, dtype, the bound's rtol, the largest ``|d| / scale``
observed ("max_rel") and the largest ``|d| / bound`` ("max_ratio"; the check
fails above 1).
"""

from __future__ import annotations

import json
import os

import numpy as np

F32, F16, F64 = "f32", "f16", "f64"
RTOL = {F32: 1e-5, F16: 1e-3, F64: 1e-12}
OUT_ROUND = {F16: 2.0 ** -11}
FLOOR = {F16: 2.0 ** -25, F32: 1e-30, F64: 0.0}


def check(got, ref, scale, *, case, family, dtype, out_dtype=None, rtol=None, floor=None,
          u_mult=1.0):
    """Assert the bound above element by element; log the observed errors.

    ``dtype`` names the arithmetic (f32 / f16 with f32 accumulation / f64) and
    sets rtol; ``out_dtype`` (default: ``dtype``) sets the output rounding and
    the floor.  ``scale`` is an array broadcastable to ``ref`` (or None for a
    plain relative bound, scale = |ref|).  ``u_mult`` scales the output
    rounding term (2 when both sides of the comparison were rounded).
    """
    out_dtype = out_dtype or dtype
    ref = np.asarray(ref, dtype=np.float64)
    got = np.asarray(got, dtype=np.float64).reshape(ref.shape)
    scale = np.abs(ref) if scale is None else np.broadcast_to(np.asarray(scale, np.float64),
                                                               ref.shape)
    rt = RTOL[dtype] if rtol is None else rtol
    fl = FLOOR[out_dtype] if floor is None else floor
    u = u_mult * OUT_ROUND.get(out_dtype, 0.0)
    err = np.abs(got - ref)
    bound = rt * scale + u * np.abs(ref) + fl
    with np.errstate(divide="ignore", invalid="ignore"):
        rel = np.where(scale > 0, err / np.where(scale > 0, scale, 1.0),
                       np.where(err > 0, np.inf, 0.0))
        ratio = np.where(bound > 0, err / np.where(bound > 0, bound, 1.0),
                         np.where(err > 0, np.inf, 0.0))
    entry = {"case": case, "family": family, "dtype": dtype, "out_dtype": out_dtype, "rtol": rt,
             "n": int(err.size), "max_rel": float(np.nanmax(rel)) if rel.size else 0.0,
             "max_ratio": float(np.nanmax(ratio)) if ratio.size else 0.0}
    log = os.environ.get("EMMY_PARITY_LOG")
    if log:
        with open(log, "a") as f:
            f.write(json.dumps(entry) + "\n")
    bad = ~(err <= bound)                      # NaN in got counts as outside
    if bad.any():
        i = np.unravel_index(int(np.argmax(np.where(bad, np.nan_to_num(ratio, nan=np.inf), -1.0))),
                             err.shape) if err.ndim else ()
        raise AssertionError(
            f"{case}: {int(bad.sum())} of {err.size} elements outside |d| <= {rt:g}*scale"
            f" + {u:g}*|ref| + {fl:g}; worst at {i}: got {got[i]!r} want {ref[i]!r}"
            f" scale {scale[i]!r}; max |d|/scale {entry['max_rel']:.3g}")
    return entry
