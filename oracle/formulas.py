"""TEST INFRASTRUCTURE ONLY -- float64 closed forms of each kernel family.

These restate what each family computes, in float64 numpy, then cast to the
output dtype.  They are the "torch-CPU evaluation" in closed form and the
strongest pin the oracle has: cast to f32 they reproduce the reference's
golden ``expected.npz`` files bit for bit (checked in ``tests/``).  Only
``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU legs use them.

Family semantics follow the IR shapes of the reference fixtures (reference
``tests/variants/*/*.ir.json``) and the elementwise spellings of
``ptxc/expr.py:880-1089``:

* rmsnorm  ``y = x * recip(sqrt(eps + sum(x*x) * recip(n))) * w``  (``v_f_rms_512``)
* l2norm   ``y = x * recip(sqrt(sum(x*x)))``                        (``v_f_l2_256``)
* softmax  ``y = exp(x - max) * recip(sum exp(x - max))``           (``v_f_softmax_1024``)
* layernorm ``y = (x - mean) * recip(sqrt(var + eps)) * g + b``     (spec ``tools/specs/ln_specs.py:2-6``)
* reductions: sum / mean / max over one axis                          (``v_r_*``, ``w_r_*``)
* matmul / bmm: ``C = A @ B`` (+ bias, relu epilogue)                 (``v_m_*``, ``w_m_*``)
* attention: ``softmax(q @ kt * recip(div)) @ v``                    (``v_a_*``, ``w_a_*``)
"""

from __future__ import annotations

import numpy as np


def _f64(a):
    return np.asarray(a).astype(np.float64)


def rmsnorm(x, w, eps, out_dtype=np.float32):
    x64 = _f64(x)
    ms = (x64 * x64).mean(-1, keepdims=True)
    y = x64 / np.sqrt(ms + eps)
    if w is not None:
        y = y * _f64(w)
    return y.astype(out_dtype)


def l2norm(x, out_dtype=np.float32):
    x64 = _f64(x)
    return (x64 / np.sqrt((x64 * x64).sum(-1, keepdims=True))).astype(out_dtype)


def softmax(x, axis=-1, out_dtype=np.float32):
    x64 = _f64(x)
    m = x64.max(axis=axis, keepdims=True)
    e = np.exp(x64 - m)
    return (e / e.sum(axis=axis, keepdims=True)).astype(out_dtype)


def layernorm(x, gamma, beta, eps, out_dtype=np.float32):
    x64 = _f64(x)
    m = x64.mean(-1, keepdims=True)
    d = x64 - m
    v = (d * d).mean(-1, keepdims=True)
    y = d / np.sqrt(v + eps)
    if gamma is not None:
        y = y * _f64(gamma)
    if beta is not None:
        y = y + _f64(beta)
    return y.astype(out_dtype)


def reduce(x, axis, op, out_dtype=np.float32):
    x64 = _f64(x)
    if op == "sum":
        r = x64.sum(axis=axis)
    elif op == "mean":
        r = x64.mean(axis=axis)
    elif op == "max":
        r = x64.max(axis=axis)
    elif op == "min":
        r = x64.min(axis=axis)
    else:
        raise ValueError(op)
    return np.asarray(r).astype(out_dtype)


def matmul(a, b, bias=None, relu=False, out_dtype=np.float32):
    c = _f64(a) @ _f64(b)
    if bias is not None:
        c = c + _f64(bias)
    if relu:
        c = np.maximum(c, 0.0)
    return c.astype(out_dtype)


def matmul_abs_bound(a, b, bias=None):
    """``|A| @ |B| (+ |bias|)``: the scale of each dot product, for error bounds."""
    c = np.abs(_f64(a)) @ np.abs(_f64(b))
    if bias is not None:
        c = c + np.abs(_f64(bias))
    return c


def matvec(a, x, out_dtype=np.float64):
    return (_f64(a) @ _f64(x)).astype(out_dtype)


def attention(q, kt, v, scale_div, out_dtype=np.float32):
    """2-D fixture form: ``q[S,D]``, ``kt[D,S]``, ``v[S,Dv]``, scores divided by ``scale_div``."""
    s = (_f64(q) @ _f64(kt)) / float(scale_div)
    p = softmax(s, axis=-1, out_dtype=np.float64)
    return (p @ _f64(v)).astype(out_dtype)


def attention_bhsd(q, k, v, scale, out_dtype=np.float32):
    """Batched form: ``q, k, v [B,H,S,D]``; scores ``q @ k^T * scale``."""
    s = np.matmul(_f64(q), np.swapaxes(_f64(k), -1, -2)) * float(scale)
    p = softmax(s, axis=-1, out_dtype=np.float64)
    return np.matmul(p, _f64(v)).astype(out_dtype)


def layernorm_abs_scale(x, gamma, beta, eps):
    """``(|x| + |mean|) * rstd * |gamma| + |beta|``: the magnitude of the terms
    each layer-norm output is formed from, for error bounds (an output near
    zero because beta cancels the normalised term still carries the terms'
    rounding)."""
    x64 = _f64(x)
    m = x64.mean(-1, keepdims=True)
    d = x64 - m
    rstd = 1.0 / np.sqrt((d * d).mean(-1, keepdims=True) + eps)
    s = (np.abs(x64) + np.abs(m)) * rstd
    if gamma is not None:
        s = s * np.abs(_f64(gamma))
    if beta is not None:
        s = s + np.abs(_f64(beta))
    return s


def attention_abs_scale(q, k, v, scale):
    """``sum_j p_j |v_j|`` per output element (q, k, v ``[..., S, D]``; k not
    transposed): the convex-combination scale of each attention output, for
    error bounds."""
    s = np.matmul(_f64(q), np.swapaxes(_f64(k), -1, -2)) * float(scale)
    p = softmax(s, axis=-1, out_dtype=np.float64)
    return np.matmul(p, np.abs(_f64(v)))
