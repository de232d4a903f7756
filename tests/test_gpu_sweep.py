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
    rd, cnt = sweep.run_device(op, bits)
    d = sweep.host_rows(rd)
    M = (1 << (bits - 1)) - 1
    for a, want in zip(g["sample_a"], g["sample_digests"]):
        assert int(d[a + M]) == want, (op, bits, a)
    assert sweep.digest(d) == g["sha"]
    cnt = cnt.cpu().numpy()
    for i, name in enumerate(("overflow", "underflow", "divide", "invalid")):
        assert int(cnt[i]) == g[f"n_{name}"], (op, bits, name)


@pytest.mark.parametrize("op", sweep.OPS)
def test_sf16_rows_match_the_oracle(gpu, op, rng):
    M = 32767
    rows = sorted(set(rng.integers(-M, M + 1, 6).tolist()) | {-M, -1, 0, 1, M})
    want, _ = oracle_rows(op, 16, rows)
    for a, wd in zip(rows, want):
        rd, _ = sweep.run_device(op, 16, a, a + 1)
        assert int(sweep.host_rows(rd)[0]) == int(wd), (op, a)


def test_row_ranges_compose(gpu):
    M = 127
    full_d, full_n = sweep.run_device("div", 8)
    parts = [(-M, -40), (-40, -40), (-40, 3), (3, M + 1)]
    ds, n = [], 0
    for lo, hi in parts:
        rd, cnt = sweep.run_device("div", 8, lo, hi)
        ds.append(rd.cpu())
        n += int(cnt[2])
    import torch
    assert torch.equal(torch.cat(ds), full_d.cpu())
    assert n == int(full_n[2]) == 255


def test_sweep_argument_errors(gpu):
    import torch
    z = torch.zeros(10, dtype=torch.int32, device="cuda")
    cnt = torch.zeros(8, dtype=torch.int64, device="cuda")
    with pytest.raises(ValueError):
        _lib.sweep("fma", 8, 0, 1, z, cnt)
    with pytest.raises(Exception):
        _lib.sweep("add", 8, -200, 0, z, cnt)
    with pytest.raises(Exception):
        _lib.sweep("add", 17, 0, 1, z, cnt)
