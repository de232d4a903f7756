"""The general chain with K split across CTAs (sfb_chain.cu: chain_piece_kernel
summarises each piece of K, chain_combine_kernel composes the pieces in
order), emulated on the CPU, against the oracle's sequential chain.

Each step v -> clip(v + t, -M, M) is a clamp-add map and a run of them is
v -> clip(v + s, lo, hi) with lo / hi the run's images of -inf / +inf; the
run leaves [-M, M] from entry v exactly when v + P does for some prefix sum P,
so the whole chain from 0 overflows when a prefix of the unclipped sum does
(pmax > M or pmin < -M, composed as s_before + the piece's pmax / pmin); a
product that truncates to 0 adds 0 and never saturates, so underflow is an OR
over the pieces.  Any cut of K into pieces must give the sequential chain's
codes and both event masks."""
import numpy as np
import pytest

from oracle import sfref

BIG = 1 << 30


def piece_summary(bits, A, B, k0, k1):
    """(s, lo, hi, pmax, pmin, under) per output for steps k0..k1-1, as
    chain_piece_kernel accumulates them."""
    Mx, S = sfref.consts(bits)
    sh = bits - 1
    M, N = A.shape[0], B.shape[1]
    s = np.zeros((M, N), np.int64)
    lo = np.full((M, N), -BIG, np.int64)
    hi = np.full((M, N), BIG, np.int64)
    pmax = np.full((M, N), -BIG, np.int64)
    pmin = np.full((M, N), BIG, np.int64)
    um = np.full((M, N), 0xFFFFFFFF, np.int64)
    for k in range(k0, k1):
        a, b = A[:, k, None], B[None, k, :]
        p = np.abs(a) * np.abs(b)                          # < 2^30
        t = np.where((a < 0) ^ (b < 0), -(p >> sh), p >> sh)
        um = np.minimum(um, (p - 1) & 0xFFFFFFFF)           # unsigned p - 1: a zero product never counts
        s += t
        pmax = np.maximum(pmax, s)
        pmin = np.minimum(pmin, s)
        lo = np.clip(lo + t, -Mx, Mx)
        hi = np.clip(hi + t, -Mx, Mx)
    return s, lo, hi, pmax, pmin, um < (1 << sh) - 1


def combine(bits, pieces):
    """chain_combine_kernel: the pieces composed in order from v = 0."""
    Mx, _ = sfref.consts(bits)
    shape = pieces[0][0].shape
    s = np.zeros(shape, np.int64)
    lo = np.full(shape, -(1 << 62), np.int64)
    hi = np.full(shape, 1 << 62, np.int64)
    pmax = np.full(shape, -(1 << 62), np.int64)
    pmin = np.full(shape, 1 << 62, np.int64)
    under = np.zeros(shape, bool)
    for bs, blo, bhi, bpmax, bpmin, bund in pieces:
        empty = bpmax == -BIG                               # an empty piece is the identity
        nlo = np.clip(lo + bs, blo, bhi)
        nhi = np.clip(hi + bs, blo, bhi)
        lo = np.where(empty, lo, nlo)
        hi = np.where(empty, hi, nhi)
        pmax = np.where(empty, pmax, np.maximum(pmax, s + bpmax))
        pmin = np.where(empty, pmin, np.minimum(pmin, s + bpmin))
        s = np.where(empty, s, s + bs)
        under |= np.where(empty, False, bund)
    v = np.clip(s, lo, hi)
    return v, (pmax > Mx) | (pmin < -Mx), under


@pytest.mark.parametrize("bits", [16, 12, 8, 5, 4])
def test_any_cut_of_k_composes_to_the_sequential_chain(bits, rng):
    Mx, _ = sfref.consts(bits)
    M, N, K = 12, 10, 120
    A = rng.integers(-Mx, Mx + 1, (M, K))
    B = rng.integers(-Mx, Mx + 1, (K, N))
    A[:3] = rng.integers(-3, 4, (3, K))                     # rows that stay small and underflow
    B[:, :2] = rng.integers(-Mx // 4, Mx // 4 + 1, (K, 2))
    B[rng.choice(K, 5, replace=False), 3] = 0
    want, ev = sfref.matmul_chain(bits, A, B)
    assert ev["overflow"].any() and (~ev["overflow"]).any() and ev["underflow"].any()
    for cuts in ([0, K], [0, 1, K], [0, 37, 38, 90, K], sorted({0, K, *rng.integers(0, K, 6)}), [0, 60, 60, K]):
        pieces = [piece_summary(bits, A, B, a, b) for a, b in zip(cuts[:-1], cuts[1:])]
        v, over, under = combine(bits, pieces)
        np.testing.assert_array_equal(v, want, err_msg=str(cuts))
        np.testing.assert_array_equal(over, ev["overflow"], err_msg=str(cuts))
        np.testing.assert_array_equal(under, ev["underflow"], err_msg=str(cuts))
