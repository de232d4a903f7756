"""The sweep's fold on the CPU: the splitmix64 weights against the published
first output, and the oracle's row digests against the reference's
(tests/golden/sweep.json): every pair at sf8 and sf4, the sample rows at sf16."""
import numpy as np
import pytest

from conftest import golden
from oracle import sfref
from superfloat.python_b200 import sweep


def test_splitmix64_known_answer():
    # the first output of SplitMix64 started at state 0
    assert int(sweep.splitmix64(np.array([0], np.uint64))[0]) == 0xE220A8397B1DCDAF


def oracle_rows(op, bits, a_codes):
    M, _ = sfref.consts(bits)
    b = np.arange(-M, M + 1, dtype=np.int64)
    ka = np.repeat(np.asarray(a_codes, np.int64), b.size)
    kb = np.tile(b, len(a_codes))
    k, ev = sfref.ew(op, bits, ka, kb)
    fl = np.zeros(ka.size, np.uint64)
    for name, bit in sweep.FLAG_BITS.items():
        if name in ev:
            fl |= np.broadcast_to(ev[name], ka.shape).astype(np.uint64) * np.uint64(bit)
    rows = len(a_codes)
    d = sweep.fold_rows(np.broadcast_to(k, ka.shape).reshape(rows, -1), fl.reshape(rows, -1),
                        sweep.weights(bits), bits)
    counts = {n: int(np.count_nonzero(np.broadcast_to(m, ka.shape))) for n, m in ev.items()}
    return d, counts


@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("op", sweep.OPS)
def test_oracle_full_sweep_matches_reference(op, bits):
    g = golden("sweep.json")["widths"][str(bits)][op]
    M, _ = sfref.consts(bits)
    d, counts = oracle_rows(op, bits, np.arange(-M, M + 1))
    assert sweep.digest(d) == g["sha"]
    for name in sweep.FLAG_BITS:
        assert counts.get(name, 0) == g[f"n_{name}"], name


@pytest.mark.parametrize("op", sweep.OPS)
def test_oracle_sf16_sample_rows_match_reference(op):
    g = golden("sweep.json")["widths"]["16"][op]
    d, _ = oracle_rows(op, 16, g["sample_a"])
    assert [int(v) for v in d] == g["sample_digests"]


def test_one_wrong_pair_always_changes_a_row_digest():
    """A single wrong code or flag changes its row's digest (odd weights),
    at every position of a row, for the smallest and largest changes."""
    bits = 8
    M = 127
    w = sweep.weights(bits)
    assert (w & np.uint64(1)).all()
    rng = np.random.default_rng(5)
    codes = rng.integers(-M, M + 1, (1, 2 * M + 1))
    flags = rng.integers(0, 16, (1, 2 * M + 1)).astype(np.uint64)
    base = sweep.fold_rows(codes, flags, w, bits)[0]
    for j in range(2 * M + 1):
        for dc, dfl in ((1, 0), (-1, 0), (0, 1), (0, 8)):
            c2, f2 = codes.copy(), flags.copy()
            if dc and abs(c2[0, j] + dc) <= M:
                c2[0, j] += dc
            elif dfl:
                f2[0, j] ^= np.uint64(dfl)
            else:
                continue
            assert sweep.fold_rows(c2, f2, w, bits)[0] != base, (j, dc, dfl)
