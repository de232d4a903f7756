"""POP of a 32-bit accumulator as the tensor-core path's finish kernel does it
(sfb_wide_tc.cu, mx_pop32: 32-bit magnitudes, the e >= 16 and d >= 32 special
cases that keep every shift in range), emulated on the CPU with uint32
semantics, against the oracle's POP (round half to even on the magnitude,
saturate at M, never -0) for every shift, every width of the SF16 block and
the accumulator values where rounding, saturation and the int32 ends matter."""
import numpy as np
import pytest

from oracle import sfref


def pop32(acc, shift, F, bits):
    """mx_pop32 on one int32 accumulator: (code, over, under)."""
    M = (1 << (bits - 1)) - 1
    e = shift - F + bits - 1
    mag = (-acc) & 0xFFFFFFFF if acc < 0 else acc
    if e >= 0:
        over = mag != 0 if e >= 16 else mag > (M >> e)
        q = M if over else (mag << e) & 0xFFFFFFFF
    else:
        d = -e
        if d >= 32:
            q = 0
        else:
            fl, rem, half = mag >> d, mag & ((1 << d) - 1), 1 << (d - 1)
            q = fl + int(rem > half or (rem == half and (fl & 1) == 1))
        over = q > M
        if over:
            q = M
    under = acc != 0 and q == 0
    return (-q if acc < 0 else q), over, under


def accumulators(rng):
    v = {0, 1, -1, 2, -2, 3, -3, (1 << 31) - 1, -(1 << 31), -(1 << 31) + 1}
    for p in range(1, 31):
        for dv in (-1, 0, 1):
            v.add((1 << p) + dv)
            v.add(-(1 << p) - dv)
            v.add((3 << (p - 1)) + dv)                   # halves at every rounding position
            v.add(-(3 << (p - 1)) - dv)
    v.update(int(x) for x in rng.integers(-(1 << 31), 1 << 31, 400))
    return np.array(sorted(x for x in v if -(1 << 31) <= x < (1 << 31)), np.int64)


@pytest.mark.parametrize("F", [22, 19])
def test_pop32_equals_the_oracle_pop(F, rng):
    accs = accumulators(rng)
    for bits in range(9, 17):
        for shift in range(sfref.SHIFT_MIN, sfref.SHIFT_MAX + 1):
            want, w_over, w_under = sfref.wide_pop(bits, accs, shift, F)
            got = [pop32(int(a), shift, F, bits) for a in accs]
            np.testing.assert_array_equal([g[0] for g in got], want, err_msg=f"sf{bits} shift {shift}")
            np.testing.assert_array_equal([g[1] for g in got], w_over, err_msg=f"sf{bits} shift {shift}")
            np.testing.assert_array_equal([g[2] for g in got], w_under, err_msg=f"sf{bits} shift {shift}")
