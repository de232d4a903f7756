"""Digests of the exhaustive pair sweep, from the reference's vectorised ops.

Run where the reference tree is (its root as the argument or in SF_REFERENCE_ROOT):

    SF_CACHE_DIR=/tmp/sfcache python tests/golden/make_sweep.py [reference_root] [--procs 8]

For each width in WIDTHS and op in add / sub / mul / div, every pair of
codes (a, b) in [-M, M]^2 goes through the reference's ``vec.OPS[op]``
(src/sf/_vectorized.py, the path tools/exhaustive.py:157-162 sweeps), and
each a-row is folded into the row digest that
``superfloat.python_b200.sweep.fold_rows`` defines.  sweep.json keeps the
sha256 of all row digests, the event totals, and the row digests of a few
sample rows.  About 5 minutes for sf16 on 8 processes.
"""
from __future__ import annotations

import json
import multiprocessing as mp
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from superfloat.python_b200 import sweep  # noqa: E402

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
from _refroot import reference_root  # noqa: E402

WIDTHS = (16, 8, 4)
SAMPLE_ROWS = 8


def _work(args):
    ref, bits, op, r0, r1 = args
    sys.path.insert(0, os.path.join(ref, "src"))
    from sf import _vectorized as vec          # the reference
    from sf._format import FORMATS
    fmt = FORMATS[bits]
    M = fmt.max_code
    n = 2 * M + 1
    codes = np.arange(-M, M + 1, dtype=np.int64)
    w = sweep.weights(bits)
    dg = np.empty(r1 - r0, np.uint32)
    counts = dict.fromkeys(sweep.FLAG_BITS, 0)
    step = max(1, (1 << 22) // n)
    for s in range(r0, r1, step):
        e = min(r1, s + step)
        ka = np.repeat(codes[s:e], n)
        kb = np.tile(codes, e - s)
        rk, rev = vec.OPS[op](fmt, ka, kb)
        fl = np.zeros(ka.size, np.uint64)
        for name, bit in sweep.FLAG_BITS.items():
            m = rev.get(name)
            if m is not None:
                m = np.broadcast_to(m, ka.shape)
                fl |= m.astype(np.uint64) * np.uint64(bit)
                counts[name] += int(np.count_nonzero(m))
        dg[s - r0:e - r0] = sweep.fold_rows(np.broadcast_to(rk, ka.shape).reshape(e - s, n), fl.reshape(e - s, n),
                                            w, bits)
    return r0, dg, counts


def main(argv):
    ref = None
    procs = 8
    args = list(argv)
    if "--procs" in args:
        i = args.index("--procs")
        procs = int(args[i + 1])
        del args[i:i + 2]
    ref = reference_root(args[0] if args else None)
    os.environ.setdefault("SF_CACHE_DIR", "/tmp/sf_cache_golden")
    out = {"source": "reference src/sf/_vectorized.py OPS over every code pair",
           "fold": "row digests of superfloat.python_b200.sweep.fold_rows; sha256 of the little-endian uint32 "
                   "row digests, rows a = -M..M",
           "widths": {}}
    ctx = mp.get_context("spawn")
    with ctx.Pool(procs) as pool:
        for bits in WIDTHS:
            M = (1 << (bits - 1)) - 1
            n = 2 * M + 1
            out["widths"][str(bits)] = {}
            for op in sweep.OPS:
                t0 = time.time()
                cuts = np.linspace(0, n, procs * 4 + 1).astype(int)
                jobs = [(ref, bits, op, int(cuts[i]), int(cuts[i + 1])) for i in range(len(cuts) - 1)
                        if cuts[i + 1] > cuts[i]]
                dg = np.empty(n, np.uint32)
                tot = dict.fromkeys(sweep.FLAG_BITS, 0)
                for r0, d, cnt in pool.imap_unordered(_work, jobs):
                    dg[r0:r0 + d.size] = d
                    for k, v in cnt.items():
                        tot[k] += v
                rows = np.linspace(0, n - 1, SAMPLE_ROWS).astype(int)
                out["widths"][str(bits)][op] = {
                    "pairs": n * n, "sha": sweep.digest(dg),
                    **{f"n_{k}": v for k, v in tot.items()},
                    "sample_a": [int(r) - M for r in rows], "sample_digests": [int(dg[r]) for r in rows]}
                print(f"sf{bits} {op}: {n * n:,} pairs in {time.time() - t0:.0f}s", flush=True)
    with open(os.path.join(HERE, "sweep.json"), "w") as f:
        json.dump(out, f, indent=1)
    print("wrote sweep.json")


if __name__ == "__main__":
    main(sys.argv[1:])
