"""The proven-mode chain kernel's packed arithmetic (sfb_chain.cu,
chain_pk_kernel), emulated on the CPU word for word, against the oracle's
sequential chain:

* two outputs (n, n+1) share one 32-bit accumulator as two 16-bit lanes;
* per lane, u = |a| (|b| << (17 - N)) + (0x7FFF + [a == 0]) << 16, upper half,
  so u = t + c with t the truncated product magnitude;
* the step adds u, or 0xFFFF - u for a negative product (a's sign as a full
  word mask, b's as a per-lane mask), with an IMAD-style wrapping add;
* each 32-k tile subtracts popc(w_a ^ w_b) per lane (w_a: a <= 0, w_b: b < 0),
  the accumulator starts at -tiles 32 0x7FFF (1 + 2^16), and the word decodes
  as lo = int16(low half), hi = (word - lo) >> 16;
* underflow of a lane: bit 15 of (u | [b == 0] 0xFFFF) was clear for some k.

The inputs satisfy the proof the kernel relies on (the oracle's L1 bound on
every partial sum is within the width), so the chain never clips and the
packed result must equal the oracle's codes and underflow masks exactly."""
import numpy as np
import pytest

from oracle import sfref

U32 = np.uint64(0xFFFFFFFF)


def emulate_pk(bits, A, B):
    """Codes (M, N) and underflow mask of chain_pk_kernel, lane pairs over N."""
    M, K = A.shape
    N = B.shape[1]
    Np = N + (N & 1)
    nk = (K + 31) // 32
    Kp = nk * 32
    Ap = np.zeros((M, Kp), np.int64)
    Ap[:, :K] = A
    Bp = np.zeros((Kp, Np), np.int64)
    Bp[:K, :N] = B
    am = np.abs(Ap).astype(np.uint64)
    ad = (np.uint64(0x7FFF) + (Ap == 0).astype(np.uint64)) << np.uint64(16)
    asg = np.where(Ap < 0, U32, np.uint64(0))
    bm = (np.abs(Bp) << (17 - bits)).astype(np.uint64)
    lo_n, hi_n = slice(0, Np, 2), slice(1, Np, 2)
    bs = np.where(Bp[:, lo_n] < 0, 0xFFFF, 0).astype(np.uint64) | np.where(Bp[:, hi_n] < 0, 0xFFFF0000, 0).astype(np.uint64)
    bz = np.where(Bp[:, lo_n] == 0, 0xFFFF, 0).astype(np.uint64) | np.where(Bp[:, hi_n] == 0, 0xFFFF0000, 0).astype(np.uint64)
    wa = (Ap <= 0)
    wb = (Bp < 0)

    acc0 = (-(nk * 32 * 0x7FFF * 0x10001)) & 0xFFFFFFFF
    acc = np.full((M, Np // 2), acc0, np.uint64)
    uf = np.full((M, Np // 2), 0xFFFFFFFF, np.uint64)
    for kt in range(nk):
        for k in range(kt * 32, kt * 32 + 32):
            plo = (am[:, k, None] * bm[None, k, lo_n] + ad[:, k, None]) & U32
            phi = (am[:, k, None] * bm[None, k, hi_n] + ad[:, k, None]) & U32
            pk2 = (plo >> np.uint64(16)) | (phi & np.uint64(0xFFFF0000))      # byte permute 0x7632
            acc = (acc + (pk2 ^ asg[:, k, None] ^ bs[None, k])) & U32
            uf &= pk2 | bz[None, k]
        ks = slice(kt * 32, kt * 32 + 32)
        nlo = (wa[:, None, ks] ^ wb.T[None, lo_n, ks]).sum(axis=2).astype(np.uint64)
        nhi = (wa[:, None, ks] ^ wb.T[None, hi_n, ks]).sum(axis=2).astype(np.uint64)
        acc = (acc - nlo - (nhi << np.uint64(16))) & U32
    word = acc.astype(np.int64)
    word = np.where(word >= 1 << 31, word - (1 << 32), word)                  # int32
    lo = ((word & 0xFFFF) ^ 0x8000) - 0x8000
    hi = (word - lo) >> 16
    codes = np.empty((M, Np), np.int64)
    codes[:, lo_n], codes[:, hi_n] = lo, hi
    under = np.empty((M, Np), bool)
    under[:, lo_n] = ((uf >> np.uint64(15)) & np.uint64(1)) == 0
    under[:, hi_n] = ((uf >> np.uint64(31)) & np.uint64(1)) == 0
    return codes[:, :N], under[:, :N]


def proven_codes(rng, bits, M, K, N):
    """Codes whose L1 bound keeps every partial sum inside the width.  The
    first half of A's rows and of B's columns hold magnitudes near the limit
    (no product truncates to 0 there); the rest mix in zeros, ones and
    products that truncate to 0."""
    Mx, S = sfref.consts(bits)
    lim = max(2, int(np.sqrt(Mx * S / K)))
    A = rng.integers(-lim, lim + 1, (M, K))
    B = rng.integers(-lim, lim + 1, (K, N))
    for X in (A[M // 2:], B[:, N // 2:]):
        flat = X.reshape(-1).copy()
        idx = rng.choice(flat.size, flat.size // 8, replace=False)
        flat[idx] = rng.choice([0, 1, -1, 2, -3], idx.size)
        X[...] = flat.reshape(X.shape)
    def big(shape):                                  # magnitudes in [0.8 lim, lim], either sign
        return rng.integers(-(-4 * lim // 5), lim + 1, shape) * rng.choice([-1, 1], shape)

    A[:M // 2] = big((M // 2, K))
    B[:, :N // 2] = big((K, N // 2))
    # zeros inside the clean block: a product a 0 or b 0 is exact, never an underflow
    A[0, rng.choice(K, 3, replace=False)] = 0
    B[rng.choice(K, 3, replace=False), 0] = 0
    assert sfref.chain_bound(bits, A, B) <= Mx
    return A, B


@pytest.mark.parametrize("bits,M,K,N", [(16, 24, 96, 40), (16, 16, 77, 33), (12, 20, 64, 18), (8, 12, 45, 15),
                                        (5, 10, 9, 7), (4, 8, 4, 5)])
def test_packed_lanes_equal_the_sequential_chain(bits, M, K, N, rng):
    A, B = proven_codes(rng, bits, M, K, N)
    want, ev = sfref.matmul_chain(bits, A, B)
    assert not ev["overflow"].any()
    got, under = emulate_pk(bits, A, B)
    np.testing.assert_array_equal(got, want)
    np.testing.assert_array_equal(under, ev["underflow"])
    assert ev["underflow"].any() and (~ev["underflow"]).any()       # both outcomes exercised
    assert not ev["underflow"][0, 0] and not ev["underflow"][1, 0]  # zeros in the clean block
