"""Generates tests/golden/math_sweep.json from the REFERENCE's pinned
functions (code/cis2-fp/gpu/cis2_math.h), evaluated by oracle/_ref/refmath
(compiled from the reference sources by `make -C oracle ref`) over the
242,428 points of oracle/math_sweep.h.  Run in the build container:

    python tests/golden/make_math_golden.py

The fixture keeps digests rather than the 6.8 MB table:
- the digest of the inputs;
- per function, the digest of the outputs with NaNs canonicalised, and the digest of the NaN index set;
- a few hundred exact rows.
The tests recompute the same digests from the oracle port (CPU) and from
the device kernels (GPU).
"""
from __future__ import annotations

import json
import os
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
import pyoracle  # noqa: E402


def main() -> None:
    exe = os.path.join(ROOT, "oracle", "_ref", "refmath")
    if not os.path.exists(exe):
        subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle"), "ref"], check=True)
    with tempfile.TemporaryDirectory() as td:
        out = os.path.join(td, "sweep.bin")
        subprocess.run([exe, out], check=True)
        x, outs = pyoracle.read_refmath(out)
    fix = pyoracle.sweep_digests(x, outs)
    fix["source"] = "reference code/cis2-fp/gpu/cis2_math.h via oracle/_ref/refmath"
    rows = sorted(set(range(0, 64)) | set(range(64, x.size, 1013)))
    fix["rows"] = [[int(x.view(np.uint32)[i])] + [int(outs[f].view(np.uint32)[i]) for f in pyoracle.MATH_FUNCS]
                   for i in rows]
    fix["row_index"] = rows
    with open(os.path.join(HERE, "math_sweep.json"), "w") as f:
        json.dump(fix, f, indent=0)
    print(f"math_sweep.json: {x.size} points, {len(rows)} exact rows")


if __name__ == "__main__":
    main()
