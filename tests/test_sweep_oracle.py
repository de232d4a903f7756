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
    dc, df = sweep.fold_rows(np.broadcast_to(k, ka.shape).reshape(rows, -1), fl.reshape(rows, -1),
                             sweep.weights(bits))
    counts = {n: int(np.count_nonzero(np.broadcast_to(m, ka.shape))) for n, m in ev.items()}
    return dc, df, counts


@pytest.mark.parametrize("bits", [8, 4])
@pytest.mark.parametrize("op", sweep.OPS)
def test_oracle_full_sweep_matches_reference(op, bits):
    g = golden("sweep.json")["widths"][str(bits)][op]
    M, _ = sfref.consts(bits)
    dc, df, counts = oracle_rows(op, bits, np.arange(-M, M + 1))
    assert sweep.digest(dc, df) == g["sha"]
    for name in sweep.FLAG_BITS:
        assert counts.get(name, 0) == g[f"n_{name}"], name


@pytest.mark.parametrize("op", sweep.OPS)
def test_oracle_sf16_sample_rows_match_reference(op):
    g = golden("sweep.json")["widths"]["16"][op]
    dc, df, _ = oracle_rows(op, 16, g["sample_a"])
    assert [int(v) for v in dc] == g["sample_codes"]
    assert [int(v) for v in df] == g["sample_flags"]
