"""The proven (clip-free) chain kernel behind sfb_linear_chain, bit for bit
against the oracle: codes, per-output flags and event counts, the bias add,
and the float64 dequantization, over widths, ragged shapes, zero-heavy and
sign-heavy operands."""
import numpy as np
import pytest

from oracle import native, sfref
from superfloat.python_b200 import _lib

pytestmark = pytest.mark.gpu


def proven_operands(bits, R, K, N, rng, zero_frac=0.1, neg_frac=0.5):
    """Codes whose L1 bound proves that no partial sum saturates."""
    M, S = sfref.consts(bits)
    B = rng.integers(0, M + 1, (K, N)) * np.where(rng.random((K, N)) < neg_frac, -1, 1)
    B[rng.random((K, N)) < zero_frac] = 0
    lim = max(1, (2 * S) // max(1, K))
    A = rng.integers(0, lim + 1, (R, K)) * np.where(rng.random((R, K)) < neg_frac, -1, 1)
    A[rng.random((R, K)) < zero_frac] = 0
    if R > 2 and K > 0:
        A[0] = 0                                     # one large code alone in its row
        A[0, rng.integers(0, K)] = -M
        A[1] = rng.integers(0, 3, K) * np.where(rng.random(K) < 0.5, -1, 1)   # tiny codes: underflow
    while sfref.chain_bound(bits, A, B) > M:
        A = np.trunc(A / 2).astype(np.int64)
    return A, B


def run_linear(bits, A, B, bias=None, a=1.0, s_col=None):
    import torch
    R, K = A.shape
    N = B.shape[1]
    dev = "cuda"
    X = torch.as_tensor(A, dtype=torch.int16, device=dev).contiguous()
    WT = torch.as_tensor(B, dtype=torch.int16, device=dev).contiguous()
    kb = None if bias is None else torch.as_tensor(bias, dtype=torch.int16, device=dev)
    sc = torch.as_tensor(s_col if s_col is not None else np.ones(N), dtype=torch.float64, device=dev)
    codes = torch.empty(R, N, dtype=torch.int16, device=dev)
    flags = torch.empty(R, N, dtype=torch.uint8, device=dev)
    y64 = torch.empty(R, N, dtype=torch.float64, device=dev)
    cnt = torch.zeros(_lib.N_COUNTS, dtype=torch.int64, device=dev)
    _lib.linear_chain(bits, X, WT, kb, a, sc, True, None, y64, codes, flags, cnt, R, N, K, max(K, 1), max(N, 1))
    torch.cuda.synchronize()
    return codes.cpu().numpy(), flags.cpu().numpy(), y64.cpu().numpy(), cnt.cpu().numpy()


def check(bits, A, B, bias=None, a=1.0, s_col=None):
    M, S = sfref.consts(bits)
    assert sfref.chain_bound(bits, A, B) <= M
    if A.shape[1]:
        want, ev = native.matmul_chain(bits, A, B)
        over, under = ev["overflow"], ev["underflow"]
    else:
        want = np.zeros((A.shape[0], B.shape[1]), np.int64)
        over = under = np.zeros(want.shape, bool)
    assert not over.any()
    if bias is not None:
        want, ev = sfref.add(bits, want, np.broadcast_to(bias, want.shape))
        over = ev["overflow"]
    codes, flags, y64, cnt = run_linear(bits, A, B, bias, a, s_col)
    np.testing.assert_array_equal(codes, want)
    np.testing.assert_array_equal((flags & 1) != 0, over)
    np.testing.assert_array_equal((flags & 2) != 0, under)
    assert int(cnt[0]) == int(over.sum()) and int(cnt[1]) == int(under.sum())
    assert int(cnt[5]) == 0 and int(cnt[6]) == 0
    sc = np.ones(B.shape[1]) if s_col is None else s_col
    np.testing.assert_array_equal(y64, want / S * a * sc)


SHAPES = [(1, 1, 1), (3, 5, 1), (7, 33, 3), (128, 32, 128), (129, 31, 127), (130, 100, 258), (5, 768, 9),
          (257, 3072, 130), (64, 2, 1000), (9, 0, 11)]


@pytest.mark.parametrize("bits", [16, 15, 12, 9, 8, 5, 4])
def test_proven_chain_shapes(bits, rng):
    for (R, K, N) in SHAPES:
        A, B = proven_operands(bits, R, K, N, rng)
        check(bits, A, B)


@pytest.mark.parametrize("bits", [16, 8])
def test_proven_chain_all_negative_all_zero_and_bias(bits, rng):
    M, S = sfref.consts(bits)
    for zf, nf in ((0.0, 1.0), (0.9, 0.5), (0.0, 0.0), (0.5, 1.0)):
        A, B = proven_operands(bits, 70, 200, 90, rng, zero_frac=zf, neg_frac=nf)
        bias = rng.integers(-M, M + 1, 90)
        s_col = rng.uniform(0.5, 2.0, 90)
        check(bits, A, B, bias=bias, a=0.37, s_col=s_col)
    A = np.zeros((40, 64), np.int64)
    B = rng.integers(-M, M + 1, (64, 40))
    check(bits, A, B)


def test_proven_chain_full_range_products(rng):
    """One nonzero per row at full scale: the largest products, t up to M - 1."""
    bits = 16
    M, S = sfref.consts(bits)
    R, K, N = 150, 96, 140
    A = np.zeros((R, K), np.int64)
    A[np.arange(R), rng.integers(0, K, R)] = rng.choice([M, -M, M - 1, 1, -1, S // 2], R)
    B = rng.choice([M, -M, 1, -1, 0, 2, S // 2, -(S // 2)], (K, N))
    B[np.arange(K), rng.integers(0, N, K)] = M
    check(bits, A, B)


def test_proven_chain_large(rng):
    """A GPT-2-sized projection against the C oracle on a row sample."""
    bits = 16
    R, K, N = 1024, 768, 2304
    A, B = proven_operands(bits, R, K, N, rng, zero_frac=0.01)
    codes, flags, _, cnt = run_linear(bits, A, B)
    rows = rng.choice(R, 48, replace=False)
    want, ev = native.matmul_chain(bits, A[rows], B)
    np.testing.assert_array_equal(codes[rows], want)
    np.testing.assert_array_equal((flags[rows] & 2) != 0, ev["underflow"])
    assert not (flags & 1).any() and int(cnt[1]) == int(((flags & 2) != 0).sum())
