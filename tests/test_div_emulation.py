"""The elementwise div's quotient step, emulated on the CPU with the
kernel's float32 arithmetic (sfb_ew_ops.cuh, the div branch of ew_one):
operands exact in float32, a reciprocal off by up to one ulp either way (the
rcp.approx error) of d 2^-sh, one fused multiply-add rounding to the nearest
integer, and the remainder x - q0 d 2^-sh from a second fused multiply-add
(one float32 rounding of the exact value), whose sign corrects q0.  It must give
floor(ua 2^sh / ub) for every 0 <= ua <= ub < 2^15, ub >= 1 (ua == ub
included: the kernel clamps the dividend to the divisor so that every
saturating case goes through the same quotient), the float remainder must be
the exact integer remainder, and the full div rule built on it must equal the
oracle."""
import numpy as np
import pytest

from oracle import sfref


def udiv_emulated(ua, ub, sh, ulp):
    fx = ua.astype(np.float32)                                    # exact: < 2^15
    fd = ub.astype(np.float32)
    r = (np.float32(1.0) / fd).astype(np.float32)
    if ulp:
        r = np.nextafter(r, np.float32(np.inf if ulp > 0 else 0.0)).astype(np.float32)
    # rcp.approx(d 2^-sh) = 2^sh rcp.approx(d): scaling by a power of two is exact
    r2 = (r * np.float32(2.0 ** sh)).astype(np.float32)
    fdp = (fd * np.float32(2.0 ** -sh)).astype(np.float32)       # exact
    x = fx.astype(np.float64) * r2.astype(np.float64)             # exact product of two float32
    assert np.all(x < 2.0 ** 22)                                  # the 1.5 * 2^23 rounding bias applies
    q0 = np.rint(x).astype(np.int64)                              # the fused add of 1.5 * 2^23: nearest, ties even
    # the second fused multiply-add: x - q0 dp exactly, rounded once to float32
    exact = -q0.astype(np.float64) * fdp.astype(np.float64) + fx.astype(np.float64)
    rem_f = exact.astype(np.float32)
    rem = (ua.astype(np.int64) << sh) - q0 * ub.astype(np.int64)
    np.testing.assert_array_equal(rem_f.astype(np.float64) * 2.0 ** sh, rem)   # the float remainder is exact
    assert np.all(np.abs(rem) < ub.astype(np.int64))
    return q0 - (rem_f < 0)


def pairs(rng):
    ua, ub = [], []
    for b in range(1, 2049):                                      # every dividend for small divisors
        ua.append(np.arange(0, b + 1))
        ub.append(np.full(b + 1, b))
    b = np.arange(1, 1 << 15)
    ua.append(b)
    ub.append(b)                                                  # every ua == ub
    ua.append(np.zeros_like(b))
    ub.append(b)
    rb = rng.integers(1, 1 << 15, 4_000_000)
    ra = (rng.random(rb.size) * (rb + 1)).astype(np.int64)
    ua.append(np.minimum(ra, rb))
    ub.append(rb)
    return np.concatenate(ua).astype(np.uint32), np.concatenate(ub).astype(np.uint32)


@pytest.mark.parametrize("sh", [15, 7])
@pytest.mark.parametrize("ulp", [-1, 0, 1])
def test_quotient_step_is_exact(sh, ulp, rng):
    ua, ub = pairs(rng)
    if sh < 15:
        keep = ub < (1 << sh) + 1
        ua, ub = ua[keep], ub[keep]
    q = udiv_emulated(ua, ub, sh, ulp)
    want = (ua.astype(np.int64) << sh) // ub.astype(np.int64)
    np.testing.assert_array_equal(q, want)


@pytest.mark.parametrize("bits", [16, 8, 4])
def test_div_rule_from_the_clamped_quotient(bits, rng):
    """sign-apply(min(floor(min(|a|, max(|b|,1)) 2^sh / max(|b|,1)), M)),
    overflow = (quotient == 2^sh and b != 0), divide = (b == 0): the kernel's
    div, equal to the oracle on every pair (sf8, sf4) or a large sample (sf16)."""
    M, S = sfref.consts(bits)
    sh = bits - 1
    if bits <= 8:
        c = np.arange(-M, M + 1)
        a, b = np.repeat(c, c.size), np.tile(c, c.size)
    else:
        a = rng.integers(-M, M + 1, 3_000_000)
        b = rng.integers(-M, M + 1, a.size)
        b[::97] = 0
        a[::89] = 0
        b[::7] = np.maximum(np.abs(a[::7]), 1) * np.sign(b[::7] + 0.5)     # |a| == |b|
    ua, ub = np.abs(a), np.abs(b)
    ub1 = np.maximum(ub, 1)
    ua1 = np.minimum(ua, ub1)
    q = udiv_emulated(ua1.astype(np.uint32), ub1.astype(np.uint32), sh, 1)
    s = np.where((a < 0) != (b < 0), -1, 1)
    got = s * np.minimum(q, M)
    want, ev = sfref.div(bits, a, b)
    np.testing.assert_array_equal(got, want)
    np.testing.assert_array_equal((q == S) & (b != 0), ev["overflow"])
    np.testing.assert_array_equal(b == 0, ev["divide"])
