"""Regenerate tests/golden/wide_8192_rows512.json from the reference (CPU).

    SF_CACHE_DIR=/tmp/sfcache python tests/golden/make_wide_rows.py [reference_root]

The wide (MX v4.9.2) 8192^3 workload (``workloads.wide_square(8192, 8192,
8192, 0)``, shift 0) computed by the reference's own
``_linalg.matmul_wide_codes`` (its compiled _fastmx loop) on rows 0..511 of
A, 32 blocks of 16 rows: per block the sha256 of the little-endian int16
codes and of the bit-packed overflow / underflow masks, and the event
counts.  About a minute on 8 threads.
"""
from __future__ import annotations

import hashlib
import json
import os
import sys

import numpy as np

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
from _refroot import reference_root  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))


def sha_codes(codes) -> str:
    return hashlib.sha256(np.ascontiguousarray(codes, dtype="<i2").tobytes()).hexdigest()


def sha_mask(mask) -> str:
    return hashlib.sha256(np.packbits(np.asarray(mask, bool).ravel()).tobytes()).hexdigest()


def main(ref: str | None = None) -> None:
    ref = reference_root(ref)
    sys.path.insert(0, os.path.join(ref, "src"))
    sys.path.insert(1, REPO)
    os.environ.setdefault("SF_CACHE_DIR", "/tmp/sf_cache_golden")
    from sf import _fastmx, _linalg          # the reference
    from sf._format import FORMATS
    from superfloat.python_b200 import workloads
    assert _fastmx.available(), "the reference's compiled MX loop did not build"
    A, B = workloads.wide_square(8192, 8192, 8192, 0)
    rows, block = 512, 16
    out = {"workload": "wide_square(8192, 8192, 8192, 0), sf16, shift 0, mx v4.9.2", "rows": rows,
           "block": block, "blocks": []}
    for r0 in range(0, rows, block):
        q, ev = _linalg.matmul_wide_codes(FORMATS[16], A[r0:r0 + block], B, 0)
        out["blocks"].append({"r0": r0, "codes": sha_codes(q), "overflow": sha_mask(ev["overflow"]),
                              "underflow": sha_mask(ev["underflow"]),
                              "n_overflow": int(ev["overflow"].sum()), "n_underflow": int(ev["underflow"].sum())})
        print(r0, flush=True)
    with open(os.path.join(HERE, "wide_8192_rows512.json"), "w") as f:
        json.dump(out, f, indent=0, separators=(",", ":"))


if __name__ == "__main__":
    main(*sys.argv[1:])
