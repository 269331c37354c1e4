"""Write the reference's golden outputs as committed fixtures (run where the reference is).

Reads every fixture package of the reference's own test suite
(``tests/variants/<id>/{meta.json, expected.npz}``; the harness that checks
them is ``tools/localrun.py:111-160``) and writes, into this directory:

* ``goldens.json``: per fixture id, the tolerance pair, the output tensor's
  name, shape and dtype, every argument's name, dtype, shape and seed or
  literal ``data`` (enough to rebuild the seeded inputs), and which expected
  positions are stored;
* ``goldens.npz``: the expected output values -- all of them up to
  ``FULL_LIMIT`` elements, otherwise ``SAMPLES`` evenly spaced positions plus
  the float64 sum and sum of squares of the whole output.

The tests rebuild each fixture's IR shape with ``emmy_ir.synth``
(``tests/golden/replicas.py``), feed it the same seeded inputs and compare
against these values with the fixture's own rtol/atol, on the CPU oracle and
on the GPU kernels, without needing the reference checkout.

Usage: ``python tests/golden/make_goldens.py [VARIANTS_DIR]``; without the
argument the reference checkout is found by ``oracle/refdir.py``
(``EMMY_REFERENCE_DIR``, else a ``reference`` checkout beside this repository).
"""

from __future__ import annotations

import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
FULL_LIMIT = 8192
SAMPLES = 2048


def main(variants: Path) -> None:
    table, arrays = {}, {}
    for d in sorted(p for p in variants.iterdir() if (p / "meta.json").exists()):
        meta = json.loads((d / "meta.json").read_text())
        k = meta["kernels"][-1]
        out_name = meta["graph_outputs"][0]
        exp = np.load(d / "expected.npz")[out_name]
        flat = exp.reshape(-1)
        entry = {
            "rtol": float(meta["rtol"]), "atol": float(meta["atol"]),
            "code": meta.get("code", ""),
            "output": out_name, "shape": list(exp.shape), "dtype": str(flat.dtype),
            "args": [{kk: a[kk] for kk in ("name", "dtype", "shape", "seed", "data", "output")
                      if kk in a} for a in k["args"]],
            "kernels": len(meta["kernels"]),
        }
        if flat.size <= FULL_LIMIT:
            entry["stored"] = "full"
        else:
            idx = np.linspace(0, flat.size - 1, SAMPLES).round().astype(np.int64)
            entry["stored"] = "sampled"
            arrays[f"{d.name}__index"] = idx
            flat = flat[idx]
            full64 = exp.reshape(-1).astype(np.float64)
            entry["sum"] = float(full64.sum())
            entry["sumsq"] = float((full64 * full64).sum())
        arrays[f"{d.name}__expected"] = flat
        table[d.name] = entry
    (HERE / "goldens.json").write_text(json.dumps(table, indent=1, sort_keys=True) + "\n")
    np.savez_compressed(HERE / "goldens.npz", **arrays)
    print(f"wrote {len(table)} fixtures")


if __name__ == "__main__":
    if len(sys.argv) > 1:
        main(Path(sys.argv[1]))
    else:
        sys.path.insert(0, str(HERE.parent.parent))
        from oracle.refdir import reference_variants
        _v = reference_variants()
        if _v is None:
            sys.exit("make_goldens: no reference checkout (set EMMY_REFERENCE_DIR)")
        main(_v)
