"""The exhaustive sweep kernel against the reference's digests
(tests/golden/sweep.json): every pair of sf16, sf8 and sf4 codes for add,
sub, mul and div, plus oracle rows and row-range sharding."""
import pytest

from conftest import golden
from superfloat.python_b200 import _lib, sweep
from test_sweep_oracle import oracle_rows

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("bits", [16, 8, 4])
@pytest.mark.parametrize("op", sweep.OPS)
def test_full_sweep_matches_reference(gpu, op, bits):
    g = golden("sweep.json")["widths"][str(bits)][op]
    rc, rf, cnt = sweep.run_device(op, bits)
    dc, df = sweep.host_rows(rc, rf)
    M = (1 << (bits - 1)) - 1
    for a, c, f in zip(g["sample_a"], g["sample_codes"], g["sample_flags"]):
        assert (int(dc[a + M]), int(df[a + M])) == (c, f), (op, bits, a)
    assert sweep.digest(dc, df) == g["sha"]
    cnt = cnt.cpu().numpy()
    for i, name in enumerate(("overflow", "underflow", "divide", "invalid")):
        assert int(cnt[i]) == g[f"n_{name}"], (op, bits, name)


@pytest.mark.parametrize("op", sweep.OPS)
def test_sf16_rows_match_the_oracle(gpu, op, rng):
    M = 32767
    rows = sorted(set(rng.integers(-M, M + 1, 6).tolist()) | {-M, -1, 0, 1, M})
    want_c, want_f, _ = oracle_rows(op, 16, rows)
    for a, wc, wf in zip(rows, want_c, want_f):
        rc, rf, _ = sweep.run_device(op, 16, a, a + 1)
        dc, df = sweep.host_rows(rc, rf)
        assert (int(dc[0]), int(df[0])) == (int(wc), int(wf)), (op, a)


def test_row_ranges_compose(gpu):
    M = 127
    full_c, full_f, full_n = sweep.run_device("div", 8)
    parts = [(-M, -40), (-40, -40), (-40, 3), (3, M + 1)]
    cs, fs, n = [], [], 0
    for lo, hi in parts:
        rc, rf, cnt = sweep.run_device("div", 8, lo, hi)
        cs.append(rc.cpu())
        fs.append(rf.cpu())
        n += int(cnt[2])
    import torch
    assert torch.equal(torch.cat(cs), full_c.cpu()) and torch.equal(torch.cat(fs), full_f.cpu())
    assert n == int(full_n[2]) == 255


def test_sweep_argument_errors(gpu):
    import torch
    z = torch.zeros(10, dtype=torch.int64, device="cuda")
    cnt = torch.zeros(8, dtype=torch.int64, device="cuda")
    with pytest.raises(ValueError):
        _lib.sweep("fma", 8, 0, 1, z, z, cnt)
    with pytest.raises(Exception):
        _lib.sweep("add", 8, -200, 0, z, z, cnt)
    with pytest.raises(Exception):
        _lib.sweep("add", 17, 0, 1, z, z, cnt)
