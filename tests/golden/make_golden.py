"""Regenerate the golden fixtures under tests/golden/ from the reference.

Run where the reference tree is (its root as the argument or in SF_REFERENCE_ROOT):

    SF_CACHE_DIR=/tmp/sfcache python tests/golden/make_golden.py [reference_root]

Two kinds of fixture:

1. The reference's own golden vectors, re-emitted compactly (same cases,
   same numbers): spec/golden/{add,sub,mul,div,fma,neg,abs,sqrt}.json ->
   elementwise.json; spec/golden/{dot,sum}.json -> chain.json;
   tests/data/mx_golden.json and mx_golden_v4.8.1.json -> wide_mx.json;
   spec/golden/wide/dot_wide_shift.json -> wide_shift.json.
2. Outputs of the reference itself on seeded inputs (ref_runs.json):
   full codes and masks of small chain / wide matmuls at several widths, and
   checksums (sha256 of the little-endian int16 codes, of the bit-packed
   masks) plus event counts for the workload-sized runs.
"""
from __future__ import annotations

import hashlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from superfloat.python_b200 import workloads  # noqa: E402

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
from _refroot import reference_root  # noqa: E402


def sha_codes(codes) -> str:
    return hashlib.sha256(np.ascontiguousarray(codes, dtype="<i2").tobytes()).hexdigest()


def sha_mask(mask) -> str:
    return hashlib.sha256(np.packbits(np.asarray(mask, bool).ravel()).tobytes()).hexdigest()


def dump(name, obj):
    with open(os.path.join(HERE, name), "w") as f:
        json.dump(obj, f, separators=(",", ":"))
    print("wrote", name, os.path.getsize(os.path.join(HERE, name)), "bytes")


def main(ref: str | None = None) -> None:
    ref = reference_root(ref)
    sys.path.insert(0, os.path.join(ref, "src"))
    os.environ.setdefault("SF_CACHE_DIR", "/tmp/sf_cache_golden")
    from sf import _linalg, _vectorized as vec   # the reference
    from sf._format import FORMATS

    def load(*p):
        with open(os.path.join(ref, *p)) as f:
            return json.load(f)

    # 1. the reference's golden vectors -----------------------------------------------------
    ew = []
    for op in ("add", "sub", "mul", "div", "fma", "neg", "abs", "sqrt"):
        for c in load("spec", "golden", f"{op}.json")["cases"]:
            ew.append({"op": op, "bits": c["bits"], "in": c["in"], "out": c["out"], "event": c["event"]})
    dump("elementwise.json", {"source": "spec/golden/{op}.json", "cases": ew})

    chain = []
    for c in load("spec", "golden", "dot.json")["cases"]:
        chain.append({"op": "dot", "bits": c["bits"], "in": c["in"], "out": c["out"], "events": c["events"]})
    for c in load("spec", "golden", "sum.json")["cases"]:
        chain.append({"op": "sum", "bits": c["bits"], "in": c["in"], "out": c["out"], "events": c["events"]})
    dump("chain.json", {"source": "spec/golden/dot.json, spec/golden/sum.json", "cases": chain})

    wide = []
    for fn, mx in (("mx_golden.json", "v4.9.2"), ("mx_golden_v4.8.1.json", "v4.8.1")):
        for c in load("tests", "data", fn)["cases"]:
            wide.append({"mx": mx, "bits": c["bits"], "shift": c["shift"], "a": c["a"], "b": c["b"],
                         "out": c["out"]})
    dump("wide_mx.json", {"source": "tests/data/mx_golden.json, tests/data/mx_golden_v4.8.1.json",
                          "cases": wide})

    dws = load("spec", "golden", "wide", "dot_wide_shift.json")["cases"]
    dump("wide_shift.json", {"source": "spec/golden/wide/dot_wide_shift.json", "cases": [
        {k: c[k] for k in ("target", "bits", "kind", "a", "b", "shift", "out", "overflow", "underflow")}
        for c in dws]})

    # 2. the reference run on seeded inputs -------------------------------------------------
    runs = {"small_chain": [], "small_wide": [], "elementwise": {}, "notes":
            "outputs of the reference (sf v0.16.0) on the seeded inputs named here"}
    rng = np.random.default_rng(1234)
    for bits in (16, 12, 9, 8, 6, 4):
        M = (1 << (bits - 1)) - 1
        for (m, k, n, lim) in ((5, 19, 7, M), (9, 40, 6, M // 8 + 1), (4, 64, 33, M // 40 + 1)):
            A = rng.integers(-lim, lim + 1, (m, k))
            B = rng.integers(-M, M + 1, (k, n))
            q, ev = _linalg.matmul_codes(FORMATS[bits], A, B)
            runs["small_chain"].append({"bits": bits, "a": A.tolist(), "b": B.tolist(), "out": q.tolist(),
                                        "overflow": ev["overflow"].astype(int).tolist(),
                                        "underflow": ev["underflow"].astype(int).tolist()})
            for mx in ("v4.9.2", "v4.8.1"):
                shift = int(rng.integers(-6, 7))
                q, ev = _linalg.matmul_wide_codes(FORMATS[bits], A, B, shift, mx)
                runs["small_wide"].append({"bits": bits, "mx": mx, "shift": shift, "a": A.tolist(),
                                           "b": B.tolist(), "out": q.tolist(),
                                           "overflow": ev["overflow"].astype(int).tolist(),
                                           "underflow": ev["underflow"].astype(int).tolist()})

    # casts of host floats (asarray's input conversion), every width
    runs["cast"] = []
    crng = np.random.default_rng(99)
    for bits in (16, 12, 8, 4):
        S = 1 << (bits - 1)
        vals = np.concatenate([crng.uniform(-1.2, 1.2, 200), (np.arange(-40, 41) + 0.5) / S,
                               [0.0, -0.0, 1.0, -1.0, 1 - 2.0 ** -bits, -(1 - 2.0 ** -bits), 2.0 ** -bits,
                                -2.0 ** -bits, 2.0 ** -(bits + 1), np.inf, -np.inf, np.nan, 1e-300]])
        k, ev = vec.cast_array(FORMATS[bits], vals)
        runs["cast"].append({"bits": bits, "values": [repr(float(v)) for v in vals], "codes": k.tolist(),
                             **{e: m.astype(int).tolist() for e, m in ev.items()}})

    # the 512 x 512 chain workload, whole
    A, B = workloads.chain_square(512, 0)
    q, ev = _linalg.matmul_codes(FORMATS[16], A, B)
    runs["chain_512"] = {"seed": 0, "codes": sha_codes(q), "overflow": sha_mask(ev["overflow"]),
                         "underflow": sha_mask(ev["underflow"]),
                         "n_overflow": int(ev["overflow"].sum()), "n_underflow": int(ev["underflow"].sum())}

    # the elementwise workload generator at 2^20 (same generator as 2^26), every op
    n = 1 << 20
    x, y, z, d = workloads.elementwise(n, 0)
    for op, args in (("add", (x, y)), ("sub", (x, y)), ("mul", (x, y)), ("fma", (x, y, z)),
                     ("div", (x, d))):
        k, ev = getattr(vec, op)(FORMATS[16], *args)
        runs["elementwise"][op] = {"n": n, "seed": 0, "codes": sha_codes(k),
                                   **{f"n_{e}": int(np.count_nonzero(m)) for e, m in ev.items()},
                                   **{f"mask_{e}": sha_mask(m) for e, m in ev.items()}}

    # the wide 8192^3 workload: the first 16 rows of the output
    A, B = workloads.wide_square(8192, 8192, 8192, 0)
    rows = 16
    q, ev = _linalg.matmul_wide_codes(FORMATS[16], A[:rows], B, 0)
    runs["wide_8192_rows16"] = {"seed": 0, "rows": rows, "codes": sha_codes(q),
                                "overflow": sha_mask(ev["overflow"]), "underflow": sha_mask(ev["underflow"]),
                                "n_overflow": int(ev["overflow"].sum()),
                                "n_underflow": int(ev["underflow"].sum()),
                                "acc_safe": bool(_linalg.matmul_wide_acc_safe(FORMATS[16], A, B))}
    dump("ref_runs.json", runs)


if __name__ == "__main__":
    main(*sys.argv[1:])
