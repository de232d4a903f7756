"""The wide tensor-core path's arithmetic, emulated on the CPU with the
kernels' own bit-sliced steps (sfb_wide_tc.cu), against the oracle's SF16-block
product (a bit-by-bit walk of the partial-product rows):

* t = (a w + 80 - C) >> 8 equals (X + 1) >> 2 with X = (a w - C) / 64;
* X mod 4 = (P + 2Q) mod 4 over the low bytes, split by a's nibbles into two
  16-entry tables F(x mod 16) and G(x >> 4) of two-bit words per (k, 32-column
  word), with w's sign and the +1 folded in (prep_kernel's column bits,
  wide_rem_kernel's table build);
* prep_kernel's A records (two k per 32-bit word) and the hot loop's decode of
  them (mask, byte permutes, sign-replicating permutes, the umulhi offset);
* u for 32 products = the two-bit add of one F and one G entry with a's sign
  as an all-ones mask, and sum_k u through the kernel's carry-save bit-plane
  counters (blocks of 8 k, chunks of 32, the pending levels and the ripple of
  every second chunk), read back by the epilogue's plane weights;
* the finish kernel's accumulator E + ((((U - h) & 3) + h - U) >> 2), E =
  floor(T / 4) mod 2^32 from the GEMM, equals sum_k s t.

A change to any of these steps can be checked here before it runs on a GPU."""
import numpy as np
import pytest

from oracle import sfref

UNIT = sfref.MX_UNITS["v4.9.2"][16]
RKC = 32          # k per chunk in wide_rem_kernel
ALL = np.uint32(0xFFFFFFFF)


def _direct(am, wm, sa, sw):
    """Per (m, n, k): X, t, u and the product sign, straight from the definitions."""
    a = am[:, None, :].astype(np.int64)               # (M, 1, K)
    w = wm.T[None, :, :].astype(np.int64)             # (1, N, K)
    C = np.zeros(np.broadcast_shapes(a.shape, w.shape), np.int64)
    for i in range(6):
        C += ((a >> i) & 1) * ((w << i) & 63)
    P = a * w - C
    assert np.all(P % 64 == 0)
    X = P // 64
    neg = sa[:, None, :] ^ sw.T[None, :, :]
    r = (X + 1) & 3
    u = np.where(neg, 3 - r, r)
    return X, (X + 1) >> 2, u, neg


def _tables(wm, sw):
    """F and G tables per (k, word, entry) as (lo, hi) uint32 bit-sliced words,
    built from B's column bits as the kernel builds them."""
    K, N = wm.shape
    NW = N // 32
    y = wm & 255
    bit = np.arange(32, dtype=np.uint64)

    def plane(v):                                       # (K, N) bools -> (K, NW) uint32 words
        return (v.reshape(K, NW, 32).astype(np.uint64) << bit).sum(axis=2).astype(np.uint32)

    yp = [plane((y >> p) & 1) for p in range(8)]
    s = plane(sw)
    zero = np.zeros_like(s)

    def yb(p):
        return yp[p] if p >= 0 else zero

    def add2(x, d):
        return x[0] ^ d[0], x[1] ^ d[1] ^ (x[0] & d[0])

    tabs = []
    for half in (0, 1):                                 # 0: F over x bits 0..3, 1: G over bits 4..7
        top = 7 - 4 * half
        d = []
        for i in range(4):
            lo, hi = yb(top - i - 1), yb(top - i)
            d.append((lo, hi ^ (lo & s)))               # -d where w is negative
        start = ((ALL if half == 0 else zero) | s, s)   # F: 1 + 2 s_w (+1, or -1 = 3); G: 3 s_w
        lo_t = np.zeros((K, NW, 16), np.uint32)
        hi_t = np.zeros((K, NW, 16), np.uint32)
        for idx in range(16):
            e = start
            for i in range(4):
                if (idx >> i) & 1:
                    e = add2(e, d[i])
            lo_t[:, :, idx], hi_t[:, :, idx] = e
        tabs.append((lo_t, hi_t))
    return tabs


RTSTR8 = (32 * 4 + 1) * 8          # table entry stride in bytes (RTSTR 64-bit pairs)


def _prmt(x, sel):
    """prmt.b32 d, x, 0, sel (default mode): byte i of d is byte sel_i & 7 of
    (x, 0), replicated from that byte's top bit when sel_i has bit 3 set."""
    pool = [(x >> (8 * i)) & 0xFF for i in range(4)] + [np.zeros_like(x)] * 4
    d = np.zeros_like(x)
    for i in range(4):
        n = (sel >> (4 * i)) & 0xF
        v = pool[n & 7]
        if n & 8:
            v = np.where(v & 0x80, 0xFF, 0).astype(x.dtype)
        d |= v << (8 * i)
    return d


def test_records_decode_as_the_hot_loop_reads_them(rng):
    """prep_kernel's A records (two k per 32-bit word: byte 0 = (x & 15) | s << 7,
    byte 1 = x >> 4, bytes 2-3 the next k) read back with the hot loop's
    operations: the F / G table offsets, and a's sign as an all-ones mask."""
    codes = rng.integers(-32767, 32768, (64, 2))
    codes[:4] = [[0, -1], [32767, -32767], [-256, 255], [16, -15]]
    a = np.abs(codes) & 255
    s = (codes < 0).astype(np.uint64)
    rec16 = (a & 15).astype(np.uint64) | (s << np.uint64(7)) | ((a >> 4).astype(np.uint64) << np.uint64(8))
    r = rec16[:, 0] | (rec16[:, 1] << np.uint64(16))
    # even k: r & 0xF, prmt 0x4441, sign prmt 0x8888
    np.testing.assert_array_equal((r & np.uint64(0xF)) * RTSTR8, (a[:, 0] & 15) * RTSTR8)
    np.testing.assert_array_equal(_prmt(r, 0x4441), a[:, 0] >> 4)
    np.testing.assert_array_equal(_prmt(r, 0x8888), np.where(codes[:, 0] < 0, 0xFFFFFFFF, 0))
    # odd k: umulhi(r & 0xF0000, stride << 16), prmt 0x4443, sign prmt 0xAAAA
    umulhi = ((r & np.uint64(0xF0000)) * np.uint64(RTSTR8 << 16)) >> np.uint64(32)
    np.testing.assert_array_equal(umulhi, (a[:, 1] & 15) * RTSTR8)
    np.testing.assert_array_equal(_prmt(r, 0x4443), a[:, 1] >> 4)
    np.testing.assert_array_equal(_prmt(r, 0xAAAA), np.where(codes[:, 1] < 0, 0xFFFFFFFF, 0))


def _u_words(am, sa, tabs):
    """(u0, u1) words per (row, k, word): the kernel's hot-loop logic ops."""
    (flo, fhi), (glo, ghi) = tabs
    x = am & 255
    xl, xh = x & 15, x >> 4
    M, K = am.shape
    kk = np.arange(K)[None, :]
    f0, f1 = flo[kk, :, xl], fhi[kk, :, xl]             # (M, K, NW)
    g0, g1 = glo[kk, :, xh], ghi[kk, :, xh]
    sam = np.where(sa, ALL, np.uint32(0))[:, :, None]
    u0 = f0 ^ g0 ^ sam
    u1 = f1 ^ (f0 & g0) ^ g1 ^ sam
    return u0, u1


def _csa(s, a, b):
    return s ^ a ^ b, (s & a) | (s & b) | (a & b)


def _counters(u0, u1):
    """sum_k u per (row, column) through wide_rem_kernel's carry-save schedule."""
    M, K, NW = u0.shape
    z = np.zeros((M, NW), np.uint32)
    p1, p2, p4, p8, p16 = z.copy(), z.copy(), z.copy(), z.copy(), z.copy()
    h32, pend32, h64, pend64, h128, pend128 = z.copy(), z.copy(), z.copy(), z.copy(), z.copy(), z.copy()
    hh = [z.copy() for _ in range(8)]
    for c in range(K // RKC):
        for b in range(RKC // 8):
            k0 = c * RKC + b * 8
            a = [u0[:, k0 + j] for j in range(8)]
            w = [u1[:, k0 + j] for j in range(8)]
            p1, c2a = _csa(p1, a[0], a[1])
            p2, c4a = _csa(p2, w[0], w[1])
            p1, c2b = _csa(p1, a[2], a[3])
            p2, c4b = _csa(p2, c2a, c2b)
            p2, c4c = _csa(p2, w[2], w[3])
            p4, c8a = _csa(p4, c4a, c4b)
            p1, c2c = _csa(p1, a[4], a[5])
            p2, c4d = _csa(p2, w[4], w[5])
            p4, c8b = _csa(p4, c4c, c4d)
            p1, c2d = _csa(p1, a[6], a[7])
            p2, c4e = _csa(p2, c2c, c2d)
            p2, c4f = _csa(p2, w[6], w[7])
            p4, c8c = _csa(p4, c4e, c4f)
            p8, c16a = _csa(p8, c8a, c8b)
            c16b = p8 & c8c
            p8 = p8 ^ c8c
            p16, c32 = _csa(p16, c16a, c16b)
            if b % 2 == 0:
                pend32 = c32
                continue
            h32, c64 = _csa(h32, pend32, c32)
            pend32 = z.copy()
            if b == 1:
                pend64 = c64
                continue
            h64, c128 = _csa(h64, pend64, c64)
            pend64 = z.copy()
            if c % 2 == 0:
                pend128 = c128
                continue
            h128, cc = _csa(h128, pend128, c128)
            pend128 = z.copy()
            for lv in range(8):
                t = hh[lv] & cc
                hh[lv] = hh[lv] ^ cc
                cc = t
    assert not pend32.any() and not pend64.any()        # both levels pair up within every chunk
    planes = [p1, p2, p4, p8, p16, h32, h64, h128, pend128] + hh
    weights = [0, 1, 2, 3, 4, 5, 6, 7, 7] + list(range(8, 16))
    bit = np.arange(32, dtype=np.uint32)
    total = np.zeros((M, NW, 32), np.int64)
    for pl, wt in zip(planes, weights):
        total += ((pl[:, :, None] >> bit) & 1).astype(np.int64) << wt
    return total.reshape(M, NW * 32)


def _codes(rng, bits, shape):
    M = (1 << (bits - 1)) - 1
    c = rng.integers(-M, M + 1, shape)
    flat = c.reshape(-1)
    idx = rng.choice(flat.size, flat.size // 10, replace=False)
    flat[idx] = rng.choice([0, 1, -1, M, -M, 255, -256, 16, -15], idx.size)
    return c


@pytest.mark.parametrize("bits,M,N,K", [(16, 64, 64, 256), (16, 32, 32, 11008), (12, 48, 96, 96)])
def test_remainder_sum_and_accumulator(bits, M, N, K, rng):
    A = _codes(rng, bits, (M, K))
    B = _codes(rng, bits, (K, N))
    am, wm = sfref.mx_mags(bits, A), sfref.mx_mags(bits, B)
    sa, sw = A < 0, B < 0

    X, t, u, neg = _direct(am, wm, sa, sw)
    # the header identity: the oracle's product is (X + 1) >> 2
    t_or = sfref.mx_product16(am[:, None, :], wm.T[None, :, :], UNIT)
    np.testing.assert_array_equal(t, t_or)

    # the tables, the two-bit add and the counters give sum_k u exactly
    u0, u1 = _u_words(am, sa, _tables(wm, sw))
    bitn = np.arange(32, dtype=np.uint32)
    per_k = (((u0[..., None] >> bitn) & 1) + 2 * ((u1[..., None] >> bitn) & 1)).reshape(M, K, N)
    np.testing.assert_array_equal(per_k.transpose(0, 2, 1), u)
    U = _counters(u0, u1)
    np.testing.assert_array_equal(U, u.sum(axis=2))

    # 4 sum s t = T + 3K/2 - U, and the finish kernel's recombination from floor(T / 4) mod 2^32
    s = np.where(neg, -1, 1)
    T = (s * X).sum(axis=2) - s.sum(axis=2) // 2
    assert np.all(s.sum(axis=2) % 2 == 0)
    st = (s * t).sum(axis=2)
    h = 3 * K // 2
    np.testing.assert_array_equal(4 * st, T + h - U)
    E = (T // 4).astype(np.int64) & 0xFFFFFFFF
    E = np.where(E >= 1 << 31, E - (1 << 32), E)        # the GEMM's int32 output
    S = E + ((((U - h) & 3) + h - U) >> 2)
    np.testing.assert_array_equal(S, st)
