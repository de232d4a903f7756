"""The clip bound the wide tensor-core path relies on (sfb_wide_tc.cu,
wide_tc_finish_kernel), checked on the CPU against the oracle's MX
accumulator, which clips per chunk of 8:

* every SF16-block product has t <= floor(a w / 256) + 1, so
  sum_k |t| <= min(rowL1 colMax, rowMax colL1) / 256 + K over the
  left-aligned magnitudes (the per-output bound), and rowL1 times the largest
  colMax of a 256-column block bounds it too (the per-row shortcut);
* where the bound is at most 2^31 - 1 no partial sum can clip, so the plain
  signed sum of the products (what the tensor cores and the remainder sum
  give) is the MX accumulator; elsewhere the kernel recomputes the output
  exactly, chunk by chunk."""
import numpy as np

from oracle import sfref

LIM = (1 << 31) - 1


def test_bound_covers_the_products_and_proves_no_clip(rng):
    bits, M, N, K = 16, 12, 16, 1024
    A = rng.integers(-32767, 32768, (M, K))
    A[M // 2:] //= 64                                   # rows the bound proves clip-free
    B = rng.integers(-32767, 32768, (K, N))
    B[:, N // 2:] //= 8
    A[0] = 32767                                        # a row whose same-sign products clip
    B[:, 0] = 32767
    am, wm = sfref.mx_mags(bits, A), sfref.mx_mags(bits, B)
    unit = sfref.MX_UNITS["v4.9.2"][16]
    t = sfref.mx_product16(am[:, :, None], wm[None, :, :], unit)          # (M, K, N)
    s = np.where((A < 0)[:, :, None] ^ (B < 0)[None, :, :], -1, 1)
    plain = (s * t).sum(axis=1)
    acc, clip, _ = sfref.wide_acc(bits, A, B)

    row_l1, row_max = am.sum(axis=1), am.max(axis=1)
    col_l1, col_max = wm.sum(axis=0), wm.max(axis=0)
    bound = (np.minimum(row_l1[:, None] * col_max[None, :], row_max[:, None] * col_l1[None, :]) >> 8) + K
    assert np.all(t <= (am[:, :, None] * wm[None, :, :] >> 8) + 1)
    assert np.all(np.abs(t).sum(axis=1) <= bound)

    block_max = col_max.max()                            # N <= 256: one column block
    row_safe = ((row_l1 * block_max) >> 8) + K <= LIM
    safe = bound <= LIM
    assert row_safe.any() and np.all(safe[row_safe])      # the shortcut never claims more than the bound
    np.testing.assert_array_equal(acc[safe], plain[safe])
    assert not clip[safe].any()
    assert safe.any() and (~safe).any() and clip.any()   # both sides of the bound, and real clips
