"""The oracle pinned against the reference's golden vectors and its own runs
(CPU only).  The oracle then checks every CUDA path in the gpu tests."""
import hashlib

import numpy as np
import pytest

from conftest import golden
from oracle import native, sfref
from superfloat.python_b200 import workloads

EW = golden("elementwise.json")["cases"]
CHAIN = golden("chain.json")["cases"]
WIDE = golden("wide_mx.json")["cases"]
WSHIFT = golden("wide_shift.json")["cases"]
RUNS = golden("ref_runs.json")


def sha_codes(c):
    return hashlib.sha256(np.ascontiguousarray(c, dtype="<i2").tobytes()).hexdigest()


def sha_mask(m):
    return hashlib.sha256(np.packbits(np.asarray(m, bool).ravel()).tobytes()).hexdigest()


def _event_of(events):
    hit = [e for e in sfref.EVENTS if e in events and bool(np.asarray(events[e]))]
    assert len(hit) <= 1
    return hit[0] if hit else None


def test_elementwise_golden_vectors():
    assert len(EW) == 660 * 5 + 114 * 3
    for c in EW:
        k, ev = sfref.ew(c["op"], c["bits"], *c["in"])
        assert int(k) == c["out"], c
        assert _event_of(ev) == c["event"], c


def test_float_cast_reference_run():
    for c in golden("ref_runs.json")["cast"]:
        vals = np.array([float(v) for v in c["values"]])
        k, ev = sfref.cast_float(c["bits"], vals)
        assert k.tolist() == c["codes"]
        for e in ("overflow", "underflow", "invalid"):
            assert ev[e].astype(int).tolist() == c[e], (c["bits"], e)


def test_chain_golden_vectors():
    for c in CHAIN:
        if c["op"] == "dot":
            a, b = np.array(c["in"][0]), np.array(c["in"][1])
            k, ev = sfref.matmul_chain(c["bits"], a[None, :], b[:, None])
            k = int(k[0, 0])
            got = {e for e in ("overflow", "underflow") if ev[e][0, 0]}
        else:
            k, ev = sfref.sum_chain(c["bits"], np.array(c["in"][0]))
            k = int(k)
            got = {e for e in ("overflow",) if ev[e]}
        assert k == c["out"], c
        assert got == set(c["events"]), c


@pytest.mark.parametrize("mx", ["v4.9.2", "v4.8.1"])
def test_wide_mxref_golden(mx):
    cases = [c for c in WIDE if c["mx"] == mx]
    assert len(cases) == 240
    for c in cases:
        q, _ = sfref.matmul_wide(c["bits"], np.array(c["a"]), np.array(c["b"]), c["shift"], mx)
        assert q.tolist() == c["out"]


def test_wide_shift_arrays_golden():
    assert len(WSHIFT) == 144
    for c in WSHIFT:
        sh = c["shift"] if isinstance(c["shift"], int) else np.array(c["shift"])
        q, ev = sfref.matmul_wide(c["bits"], np.array(c["a"]), np.array(c["b"]), sh, c["target"])
        assert q.tolist() == c["out"]
        assert ev["overflow"].astype(int).tolist() == c["overflow"]
        assert ev["underflow"].astype(int).tolist() == c["underflow"]


def test_small_reference_runs():
    for c in RUNS["small_chain"]:
        q, ev = sfref.matmul_chain(c["bits"], np.array(c["a"]), np.array(c["b"]))
        assert q.tolist() == c["out"]
        assert ev["overflow"].astype(int).tolist() == c["overflow"]
        assert ev["underflow"].astype(int).tolist() == c["underflow"]
        q2, ev2 = native.matmul_chain(c["bits"], np.array(c["a"]), np.array(c["b"]))
        assert q2.tolist() == c["out"] and ev2["underflow"].astype(int).tolist() == c["underflow"]
    for c in RUNS["small_wide"]:
        for acc_fn in (None, native.wide_acc):
            q, ev = sfref.matmul_wide(c["bits"], np.array(c["a"]), np.array(c["b"]), c["shift"], c["mx"],
                                      acc_fn=acc_fn)
            assert q.tolist() == c["out"]
            assert ev["overflow"].astype(int).tolist() == c["overflow"]
            assert ev["underflow"].astype(int).tolist() == c["underflow"]


def test_chain_512_reference_checksum():
    A, B = workloads.chain_square(512, 0)
    q, ev = native.matmul_chain(16, A, B)
    r = RUNS["chain_512"]
    assert sha_codes(q) == r["codes"]
    assert sha_mask(ev["overflow"]) == r["overflow"] and sha_mask(ev["underflow"]) == r["underflow"]
    assert int(ev["overflow"].sum()) == 262144 and int(ev["underflow"].sum()) == 44287


def test_elementwise_workload_reference_checksums():
    n = 1 << 20
    x, y, z, d = workloads.elementwise(n, 0)
    args = {"add": (x, y), "sub": (x, y), "mul": (x, y), "fma": (x, y, z), "div": (x, d)}
    for op, r in RUNS["elementwise"].items():
        k, ev = sfref.ew(op, 16, *args[op])
        assert sha_codes(k) == r["codes"], op
        for e, m in ev.items():
            assert int(m.sum()) == r[f"n_{e}"] and sha_mask(m) == r[f"mask_{e}"], (op, e)


def test_elementwise_workload_shape():
    """The generator's distribution: 10% forced to |v| >= 0.9 on top of the
    uniform codes' own 8%, 10% near 0, ~1% zero divisors, ~90% |b| > |a|."""
    n = 1 << 18
    x, y, z, d = workloads.elementwise(n, 3)
    M = 32767
    assert 0.17 < np.mean(np.abs(x) >= 0.9 * 32768) < 0.19
    assert 0.09 < np.mean((np.abs(x) >= 1) & (np.abs(x) <= 127)) < 0.11
    assert 0.008 < np.mean(d == 0) < 0.012
    nz = d != 0
    assert 0.85 < np.mean(np.abs(d[nz]) > np.abs(x[nz])) < 0.93
    assert np.abs(np.concatenate([x, y, z, d])).max() <= M


@pytest.mark.slow
def test_wide_8192_rows_reference_checksum():
    """The first 16 rows of the 8192^3 wide workload, C oracle vs the reference's run."""
    r = RUNS["wide_8192_rows16"]
    A_full, B = workloads.wide_square(8192, 8192, 8192, 0)
    A = A_full[:16]
    q, ev = sfref.matmul_wide(16, A, B, 0, acc_fn=native.wide_acc)
    assert sha_codes(q) == r["codes"]
    assert int(ev["overflow"].sum()) == r["n_overflow"] and int(ev["underflow"].sum()) == r["n_underflow"]
    assert sha_mask(ev["overflow"]) == r["overflow"] and sha_mask(ev["underflow"]) == r["underflow"]


def test_oracle_matches_reference_c_accumulator():
    """oracle.c and the reference's own compiled loop agree (when oracle/_ref was built)."""
    if not native.ref_available():
        pytest.skip("oracle/_ref was not built (no reference tree at build time)")
    rng = np.random.default_rng(7)
    for bits in (16, 13, 9, 8, 5, 4):
        M = (1 << (bits - 1)) - 1
        for mx in ("v4.9.2", "v4.8.1"):
            A = rng.integers(-M, M + 1, (9, 70))
            B = rng.integers(-M, M + 1, (70, 11))
            a1, c1, _ = native.wide_acc(bits, A, B, mx)
            a2, c2, _ = native.ref_wide_acc(bits, A, B, mx)
            assert (a1 == a2).all() and (c1 == c2).all()


def test_sf16_product_closed_form_exhaustive_low_bits():
    """(a w + 80 - C) >> 8 equals the bitwise partial-product walk: every
    low-6-bit pair, on many high parts (the closed form the kernels use)."""
    u = sfref.MX_UNITS["v4.9.2"][16]
    rng = np.random.default_rng(11)
    lo = np.arange(64)
    for _ in range(8):
        ha, hw = rng.integers(0, 512, 2)
        a = (ha << 6 | lo)[:, None]
        w = (hw << 6 | lo)[None, :]
        assert (sfref.t16_closed(a, w) == sfref.mx_product16(a, w, u)).all()
    a = rng.integers(0, 32768, 1 << 16)
    w = rng.integers(0, 32768, 1 << 16)
    assert (sfref.t16_closed(a, w) == sfref.mx_product16(a, w, u)).all()


def test_oracle_wide_acc_equals_the_references_own_c_loop():
    """The oracle's C accumulator (a bit-walk restatement) against the
    reference's own compiled MX loop (oracle/_ref, built from the reference's
    source string by oracle/build_ref.py) on random 2-D problems: every width's
    block, both MX versions, full-range and clipping operands."""
    from oracle import native
    if not native.ref_available():
        pytest.skip("oracle/_ref was not built (no reference tree in this container)")
    rng = np.random.default_rng(41)
    for mx in ("v4.9.2", "v4.8.1"):
        for bits in (16, 13, 9, 8, 5, 4):
            M_ = (1 << (bits - 1)) - 1
            for (m, k, n) in ((23, 57, 19), (64, 300, 40), (8, 2400, 6)):
                A = rng.integers(-M_, M_ + 1, (m, k))
                B = rng.integers(-M_, M_ + 1, (k, n))
                A[:2] = np.abs(A[:2])                    # same-sign rows clip for real
                B[:, :2] = np.abs(B[:, :2])
                got = native.wide_acc(bits, A, B, mx)
                want = native.ref_wide_acc(bits, A, B, mx, threads=2)
                np.testing.assert_array_equal(got[0], want[0], err_msg=f"sf{bits} {mx} {m}x{k}x{n}")
                np.testing.assert_array_equal(got[1], want[1])
                assert got[2] == want[2]
                if k == 2400 and bits == 16:
                    assert got[1][:2, :2].all()            # the accumulator's limit is reached


def test_wide_rows512_fixture_agrees_with_the_rows16_run():
    """The 512-row fixture's first block is the 16-row run recorded before."""
    a = golden("wide_8192_rows512.json")["blocks"][0]
    b = golden("ref_runs.json")["wide_8192_rows16"]
    assert a["codes"] == b["codes"] and a["overflow"] == b["overflow"] and a["underflow"] == b["underflow"]
