"""The elementwise fma as the kernel computes it (sfb_ew_ops.cuh: p = a b in
32 bits, trunc(p / 2^(N-1)) by the bias-and-shift of tdiv_pow2, + c, one clamp;
underflow = small_nonzero(p), with no "and not overflow" term because a
product that truncates to 0 leaves c in range), emulated on the CPU against
the oracle's fma, exhaustively over every (a, b, c) triple of sf4 and sf8.
The exhaustive GPU sweep covers the two-operand ops; this covers the
three-operand one."""
import numpy as np
import pytest

from oracle import sfref


def fma_kernel(bits, a, b, c):
    M = (1 << (bits - 1)) - 1
    sh = bits - 1
    p = a * b                                               # |p| < 2^30: fits int32
    bias = np.where(p < 0, (1 << sh) - 1, 0)                # (p >> 31) & (2^sh - 1)
    t = (p + bias) >> sh
    s = t + c
    r = np.clip(s, -M, M)
    small = ((p + ((1 << sh) - 1)) & 0xFFFFFFFF) <= (2 << sh) - 2  # the unsigned range test
    return r, r != s, small & (p != 0)


@pytest.mark.parametrize("bits", [4, 8])
def test_fma_every_triple(bits):
    M, _ = sfref.consts(bits)
    v = np.arange(-M, M + 1, dtype=np.int64)
    a, b = np.repeat(v, v.size), np.tile(v, v.size)
    for c0 in range(-M, M + 1):
        c = np.full(a.size, c0, np.int64)
        got, over, under = fma_kernel(bits, a, b, c)
        want, ev = sfref.fma(bits, a, b, c)
        np.testing.assert_array_equal(got, want)
        np.testing.assert_array_equal(over, ev["overflow"])
        np.testing.assert_array_equal(under, ev["underflow"])
