"""Family matcher for the tiled matmul / split-K IR shape (filled in below)."""

from __future__ import annotations

from .match_reduce import NoMatch


def match_gemm(kop, tile, meta) -> dict:
    raise NoMatch("matmul family not recognised")
