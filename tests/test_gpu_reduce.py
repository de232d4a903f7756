"""Sequential saturating sum and the 1-D chain dot on the B200 (the ordered
parallel reduction of clamp-add maps) vs the reference's golden cases and the
oracle: codes and events, every layout path (strided axis, one CTA per
output, outputs split across CTAs with the second pass), ragged and
unaligned lengths, and the array API."""
import numpy as np
import pytest

from conftest import golden
from oracle import native, sfref
import superfloat.python_b200 as sf
from superfloat.python_b200 import FORMATS

pytestmark = pytest.mark.gpu


def test_reference_sum_and_dot_cases(gpu):
    for c in golden("chain.json")["cases"]:
        fmt = FORMATS[c["bits"]]
        if c["op"] == "sum":
            codes, masks = gpu.run("sum", fmt, np.array(c["in"][0]), axis=0)
            assert int(codes) == c["out"], c
            assert bool(masks["overflow"]) == ("overflow" in c["events"]), c
        else:
            a, b = np.array(c["in"][0]), np.array(c["in"][1])
            codes, masks = gpu.run("matmul", fmt, a[None, :], b[:, None])
            assert int(codes[0, 0]) == c["out"], c
            got = [e for e in ("overflow", "underflow") if masks[e][0, 0]]
            assert sorted(got) == sorted(c["events"]), c


def _codes(rng, bits, shape, big=0.3):
    M = (1 << (bits - 1)) - 1
    x = rng.integers(-M // 8, M // 8 + 1, shape)
    hot = rng.random(shape) < big
    x[hot] = rng.integers(-M, M + 1, int(hot.sum()))
    return x


@pytest.mark.parametrize("bits", [16, 12, 8, 4])
def test_sum_every_layout(gpu, bits, rng):
    fmt = FORMATS[bits]
    cases = [((7, 33, 5), 1), ((7, 33, 5), 0), ((7, 33, 5), 2), ((3, 4096), 1), ((1, 1 << 20), 1), ((2, 12345), -1),
             ((40000, 12), 1), ((5,), 0), ((9, 8, 1), 1)]
    for shape, axis in cases:
        x = _codes(rng, bits, shape)
        want, ev = sfref.sum_chain(bits, x, axis % len(shape))
        got, masks = gpu.run("sum", fmt, x, axis=axis)
        np.testing.assert_array_equal(got, want, err_msg=f"sf{bits} {shape} axis {axis}")
        np.testing.assert_array_equal(masks["overflow"], ev["overflow"], err_msg=f"sf{bits} {shape} axis {axis}")


def test_sum_long_chains_with_recoveries(gpu, rng):
    """Chains that saturate, come back and saturate again, on the split path."""
    fmt = FORMATS[16]
    M = 32767
    n = 3_000_017
    x = np.where(rng.random(n) < 0.5, 1, -1) * rng.integers(0, 40, n)
    x[1000:1100] = M                          # up to +M ...
    x[2_000_000:2_000_200] = -M               # ... down to -M, then a random walk again
    want, ev = sfref.sum_chain(16, x[:, None], 0)
    got, masks = gpu.run("sum", fmt, x, axis=0)
    assert int(got) == int(want[0]) and bool(masks["overflow"]) == bool(ev["overflow"][0])
    y = np.tile([3, -3], 100_000)                # partial sums stay in [0, 3]
    got, masks = gpu.run("sum", fmt, y, axis=0)
    assert int(got) == 0 and not masks["overflow"]


@pytest.mark.parametrize("bits", [16, 8])
def test_dot_long(gpu, bits, rng):
    fmt = FORMATS[bits]
    for n in (1, 7, 1000, 100_003, 1 << 21):
        a = _codes(rng, bits, n, big=0.05)
        b = _codes(rng, bits, n, big=0.05)
        want, ev = native.matmul_chain(bits, a[None, :], b[:, None])
        got, masks = gpu.run("matmul", fmt, a[None, :], b[:, None])
        assert int(got[0, 0]) == int(want[0, 0]), (bits, n)
        for e in ("overflow", "underflow"):
            assert bool(masks[e][0, 0]) == bool(ev[e][0, 0]), (bits, n, e)


def test_array_api_sum_and_status(gpu, rng):
    x = sf.from_codes(_codes(rng, 16, (6, 300)), sf.sf16)
    with sf.errstate(all="ignore"):
        r = sf.sum(x, axis=1)
        r2 = x.sum(axis=1)
        r3 = sf.sum(x)
    want, ev = sfref.sum_chain(16, x.codes, 1)
    assert r.codes.tolist() == want.tolist() == r2.codes.tolist()
    flat, _ = sfref.sum_chain(16, x.codes.reshape(-1), 0)
    assert int(r3.codes) == int(flat)
    small = sf.from_codes(np.arange(10) - 5, sf.sf16)
    assert int(sf.sum(small).codes) == -5
    with pytest.raises(sf.SFShapeError):
        sf.sum(x, axis=2)
