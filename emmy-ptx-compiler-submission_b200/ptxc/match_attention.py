"""Family matcher for the attention-like matmul -> softmax -> reduce IR shape."""

from __future__ import annotations

from .match_reduce import NoMatch


def match_attention(kop, tile, meta) -> dict:
    raise NoMatch("attention family not recognised")
