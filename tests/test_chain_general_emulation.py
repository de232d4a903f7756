"""CPU emulation of the general-mode chain kernel's step (chain2_kernel)
against the oracle's sequential chain, at several widths, on random and
edge codes: t = umulhi(|a| << (32 - (N-1)), |b|), the underflow minimum of
|a| |b| - 1 (unsigned 32-bit), s = t (sa sb) + acc in int32, the clip to
[-M, M] and the overflow OR of s ^ clip(s).  No GPU."""
import numpy as np
import pytest

from oracle import sfref

U32 = np.uint64(0xFFFFFFFF)


def emulate(bits, A, B):
    sh = bits - 1
    M = (1 << sh) - 1
    A = np.asarray(A, np.int64)
    B = np.asarray(B, np.int64)
    m, K = A.shape
    n = B.shape[1]
    acc = np.zeros((m, n), np.int64)
    um = np.full((m, n), 0xFFFFFFFF, np.uint64)
    ov = np.zeros((m, n), bool)
    for k in range(K):
        aa = np.abs(A[:, k]).astype(np.uint64)[:, None]
        ba = np.abs(B[k, :]).astype(np.uint64)[None, :]
        ahi = (aa << np.uint64(32 - sh)) & U32                 # a 32-bit register
        t = ((ahi * ba) >> np.uint64(32)).astype(np.int64)      # umulhi
        pm1 = (aa * ba + U32) & U32                            # IMAD with addend -1, 32-bit
        um = np.minimum(um, pm1)
        sg = np.where(A[:, k] < 0, -1, 1)[:, None] * np.where(B[k, :] < 0, -1, 1)[None, :]
        s = t * sg + acc
        assert np.abs(s).max(initial=0) < 2 ** 31              # int32 never wraps
        c = np.clip(s, -M, M)
        ov |= s != c
        acc = c
    under = um < np.uint64((1 << sh) - 1)
    return acc, ov, under


@pytest.mark.parametrize("bits", [16, 12, 8, 5, 4])
def test_step_equals_the_sequential_chain(bits):
    rng = np.random.default_rng(bits)
    M = (1 << (bits - 1)) - 1
    edges = np.array([0, 1, -1, 2, -2, M, -M, M - 1, -(M - 1), M // 2, -(M // 2)])
    for (m, K, n) in ((7, 40, 9), (5, 300, 6)):
        A = rng.integers(-M, M + 1, (m, K))
        B = rng.integers(-M, M + 1, (K, n))
        A[0] = rng.choice(edges, K)
        B[:, 0] = rng.choice(edges, K)
        A[1] = rng.integers(-3, 4, K)                          # small products: underflow
        got, ov, un = emulate(bits, A, B)
        want, ev = sfref.matmul_chain(bits, A, B)
        np.testing.assert_array_equal(got, want)
        np.testing.assert_array_equal(ov, ev["overflow"])
        np.testing.assert_array_equal(un, ev["underflow"])


def test_a_planted_mistake_is_caught():
    """Taking the high word of |a| |b| << (32 - N) (one bit short) breaks
    the products: the step is load-bearing."""
    bits = 16
    rng = np.random.default_rng(3)
    A = rng.integers(-32767, 32768, (4, 50))
    B = rng.integers(-32767, 32768, (50, 5))
    sh = bits - 1
    aa = np.abs(A).astype(np.uint64)
    ba = np.abs(B).astype(np.uint64)
    t_ok = ((((aa[:, :1] << np.uint64(32 - sh)) & U32) * ba[:1, :]) >> np.uint64(32))
    t_bad = ((((aa[:, :1] << np.uint64(31 - sh)) & U32) * ba[:1, :]) >> np.uint64(32))
    assert not np.array_equal(t_ok, t_bad)
    np.testing.assert_array_equal(t_ok, (aa[:, :1] * ba[:1, :]) >> np.uint64(sh))
