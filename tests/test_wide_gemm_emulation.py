"""The integer-linear half of the wide tensor-core path, emulated on the CPU
byte for byte: prep_kernel's nine int8 planes per operand (signed high limb h,
unsigned low limb l of the left-aligned signed code, six bit / negated-C
planes, the +-1 / -+32 sign planes), tc_gemm_kernel's eleven passes with their
signedness (D0 = h.h, D1 = h.l + l.h, D2 = l.l + the seven bit and sign
passes), the in-TMEM fold 2^8 D0 + D1 (mod 2^32) and the epilogue's + D2 >> 8.

It must give floor(T / 4) mod 2^32 with T = sum s X - (sum s) / 2 and
X = (a w - C) / 64 straight from the definitions, and every D must stay
inside int32 up to K = 16384 (the accumulators are 32-bit)."""
import numpy as np
import pytest


def planes(codes, bits, is_a):
    """The nine planes of prep_kernel as int64 values of their int8 bytes,
    read signed or unsigned as the GEMM reads them: (9, rows, K)."""
    a = np.abs(codes).astype(np.int64) << (16 - bits)
    s = codes < 0
    kt = np.where(s, -a, a)
    out = [((kt >> 8) & 0xFF).astype(np.int8).astype(np.int64),          # h, signed
           (kt & 0xFF).astype(np.int64)]                                # l, unsigned
    for i in range(6):
        v = ((a >> i) & 1) if is_a else -((a << i) & 63)
        v = np.where(s, -v, v)
        out.append((v & 0xFF).astype(np.int8).astype(np.int64))
    sg = np.where(s, -1, 1) if is_a else np.where(s, 32, -32)
    out.append((sg & 0xFF).astype(np.int8).astype(np.int64))
    return np.stack(out)


def gemm_passes(pa, pb):
    """D0, D1, D2 over K (pb is (9, N, K) with K last, as the B planes are stored)."""
    mm = lambda p, q: pa[p] @ pb[q].T                                    # noqa: E731
    D0 = mm(0, 0)
    D1 = mm(0, 1) + mm(1, 0)
    D2 = mm(1, 1) + sum(mm(p, p) for p in range(2, 9))
    return D0, D1, D2


def wrap32(x):
    x = np.asarray(x, np.int64) & 0xFFFFFFFF
    return np.where(x >= 1 << 31, x - (1 << 32), x)


def direct_T(A, B, bits):
    am = np.abs(A).astype(np.int64) << (16 - bits)
    wm = (np.abs(B).astype(np.int64) << (16 - bits)).T                 # (N, K)
    a, w = am[:, None, :], wm[None, :, :]
    C = np.zeros(np.broadcast_shapes(a.shape, w.shape), np.int64)
    for i in range(6):
        C += ((a >> i) & 1) * ((w << i) & 63)
    X = (a * w - C) // 64
    s = np.where((A < 0)[:, None, :] ^ (B < 0).T[None, :, :], -1, 1)
    return (s * X).sum(axis=2) - s.sum(axis=2) // 2


@pytest.mark.parametrize("bits,M,N,K", [(16, 8, 12, 256), (13, 6, 10, 128), (16, 4, 4, 16384)])
def test_planes_passes_and_fold_give_floor_T_over_4(bits, M, N, K, rng):
    Mx = (1 << (bits - 1)) - 1
    A = rng.integers(-Mx, Mx + 1, (M, K))
    B = rng.integers(-Mx, Mx + 1, (K, N))
    A[0], B[:, 0] = -Mx, -Mx                          # the extreme limbs (h = -128) on a whole row / column
    A[1], B[:, 1] = Mx, -Mx
    A[2, ::3] = 0
    D0, D1, D2 = gemm_passes(planes(A, bits, True), planes(B.T, bits, False))
    for D in (D0, D1, D2):
        assert np.abs(D).max() < 1 << 31
    E = wrap32(wrap32((D0 << 8) + D1) + (D2 >> 8))
    T = direct_T(A, B, bits)
    np.testing.assert_array_equal(E, wrap32(T // 4))
    assert np.all((1 << 16) * D0 + (1 << 8) * D1 + D2 == 64 * T)      # the exact identity before the cut


def test_accumulators_fit_int32_up_to_k_16384():
    """Worst case per k from the planes' ranges (h in [-128, 127], l in
    [0, 255], bit planes in {-1, 0, 1}, C planes in [-63, 63], sign planes
    +-1 x +-32), times K = 16384: every D fits a 32-bit accumulator."""
    kmax = 16384
    d0 = 128 * 128
    d1 = 2 * 128 * 255
    d2 = 255 * 255 + 6 * 63 + 32
    assert kmax * max(d0, d1, d2) < 1 << 31
