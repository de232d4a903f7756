"""The elementwise sqrt as the kernel computes it (sfb_ew_ops.cuh, the sqrt
branch of ew_one: x = max(a, 0) << (N - 1), r = (int) sqrtf((float) x), then
one step down and one step up so that r = floor(sqrt(x))), emulated on the CPU
with the same float32 rounding (the int-to-float conversion and sqrtf are both
correctly rounded), against the oracle over every code of every width.  Over
these inputs the truncated sqrtf is floor(sqrt(x)) or (at a few widths) one
above it, so only the downward step ever fires; the upward one is a guard."""
import numpy as np
import pytest

from oracle import sfref


@pytest.mark.parametrize("bits", range(4, 17))
def test_sqrt_every_code(bits):
    M, _ = sfref.consts(bits)
    a = np.arange(-M, M + 1, dtype=np.int64)
    x = np.maximum(a, 0) << (bits - 1)                              # < 2^30
    r = np.sqrt(x.astype(np.float32)).astype(np.int64)              # truncation, as the (int) cast
    assert np.all(np.abs(r - np.floor(np.sqrt(x.astype(np.float64)))) <= 1)
    down = r * r > x
    r -= down
    up = (r + 1) * (r + 1) <= x
    r += up
    assert not up.any()
    want, ev = sfref.sqrt(bits, a)
    np.testing.assert_array_equal(r, want)
    np.testing.assert_array_equal(a < 0, ev["invalid"])
