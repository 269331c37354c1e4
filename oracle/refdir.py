"""TEST INFRASTRUCTURE ONLY -- where the reference checkout is, if anywhere.

The reference repository (``titoatwork/emmy-ptx-compiler-submission``) is not
redistributable, so nothing of it is committed here; the test set-up and the
fixture generators read it in place when a checkout is available:

1. the directory named by the ``EMMY_REFERENCE_DIR`` environment variable, or
2. a checkout named ``reference`` next to this repository's root directory.

``reference_dir()`` returns that directory when it holds the reference's
``compile.py``, else ``None``; callers skip what needs the checkout when it is
absent (as on a GPU box, which only receives the files generated from it).
"""

from __future__ import annotations

import os
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent


def reference_dir() -> Path | None:
    env = os.environ.get("EMMY_REFERENCE_DIR")
    cands = [Path(env)] if env else [ROOT.parent / "reference"]
    for c in cands:
        if (c / "compile.py").is_file():
            return c
    return None


def reference_variants() -> Path | None:
    ref = reference_dir()
    if ref is None:
        return None
    v = ref / "tests" / "variants"
    return v if v.is_dir() else None
