"""The sequential saturating sum / dot as the reduction kernels compute them in
parallel (sfb_reduce.cu: chunk_seg per thread, cta_reduce's shuffle-down tree
inside each warp and the warps in order, reduce_pieces_kernel per piece of K,
combine_pieces_kernel over the pieces), emulated on the CPU against the
oracle's one-step-at-a-time chain.  The clamp-add segments must compose to
the sequential result for any piece span and chunk length, including threads
whose chunk is empty (the identity segment)."""
import numpy as np
import pytest

from oracle import sfref

RT = 256
INF = 1 << 62


def identity():
    return (0, -INF, INF, -INF, INF, 0)


def compose(A, B):
    s = A[0] + B[0]
    lo = min(max(A[1] + B[0], B[1]), B[2])
    hi = min(max(A[2] + B[0], B[1]), B[2])
    return (s, lo, hi, max(A[3], A[0] + B[3]), min(A[4], A[0] + B[4]), A[5] | B[5])


def chunk_seg(xs, under, M):
    """One thread's chunk: int running values, lo / hi started at -+2^30."""
    if len(xs) == 0:
        return identity()
    s, pmax, pmin, lo, hi = 0, -(1 << 30), 1 << 30, -(1 << 30), 1 << 30
    for x in xs:
        s += x
        pmax, pmin = max(pmax, s), min(pmin, s)
        lo = min(max(lo + x, -M), M)
        hi = min(max(hi + x, -M), M)
    return (s, lo, hi, pmax, pmin, int(under))


def cta_reduce(segs):
    """The warp shuffle-down tree (lane 0 of each warp), then the warps in order."""
    warps = []
    for w0 in range(0, RT, 32):
        v = list(segs[w0:w0 + 32])
        off = 1
        while off < 32:
            o = [v[i + off] if i + off < 32 else v[i] for i in range(32)]       # shfl_down
            v = [compose(v[i], o[i]) if (i & (2 * off - 1)) == 0 and i + off < 32 else v[i] for i in range(32)]
            off <<= 1
        warps.append(v[0])
    t = warps[0]
    for w in warps[1:]:
        t = compose(t, w)
    return t


def reduce_one(x, under_k, span, chunk, M):
    """One output's K through pieces of span and per-thread chunks."""
    K = len(x)
    pieces = []
    for base in range(0, max(K, 1), span):
        end = min(K, base + span)
        segs = []
        for t in range(RT):
            k0 = min(end, base + t * chunk)
            k1 = min(end, k0 + chunk)
            segs.append(chunk_seg(x[k0:k1], under_k[k0:k1].any(), M))
        pieces.append(cta_reduce(segs))
    t = pieces[0]
    for p in pieces[1:]:
        t = compose(t, p)
    v = min(max(t[0], t[1]), t[2])
    return v, t[3] > M or t[4] < -M, bool(t[5])


@pytest.mark.parametrize("bits", [16, 8, 4])
@pytest.mark.parametrize("span,chunk", [(4096, 16), (700, 3), (97, 1), (5000, 40)])
def test_sum_and_dot_compose_to_the_sequential_chain(bits, span, chunk, rng):
    M, S = sfref.consts(bits)
    K = 3001
    a = rng.integers(-M, M + 1, K)
    a[1000:1300] = M                                   # a saturating run
    b = rng.integers(-M, M + 1, K)
    b[::5] = rng.integers(-2, 3, b[::5].size)          # products that truncate to 0
    # sum: the values themselves, no underflow
    want, ev = sfref.sum_chain(bits, a)
    v, over, under = reduce_one(a, np.zeros(K, bool), span, chunk, M)
    assert (v, over) == (int(want), bool(ev["overflow"]))
    # no saturation, but a later run rises 1.2 M from -0.6 M: its own prefix
    # leaves the range, the true one does not (the pmax / pmin offsets matter)
    step = max(1, M // 500)
    n1, n2 = int(0.6 * M / step), int(1.2 * M / step)
    c = np.zeros(K, np.int64)
    c[:n1], c[n1:n1 + n2] = -step, step
    want, ev = sfref.sum_chain(bits, c)
    assert not ev["overflow"]
    v, over, under = reduce_one(c, np.zeros(K, bool), span, chunk, M)
    assert (v, over) == (int(want), False)
    # one-sided drifts: overflow only through accumulation across chunks, on
    # the high side and on the low side separately
    for sign in (1, -1):
        d = sign * rng.integers(0, max(2, M // 16), K)
        want, ev = sfref.sum_chain(bits, d)
        assert ev["overflow"]
        v, over, under = reduce_one(d, np.zeros(K, bool), span, chunk, M)
        assert (v, over) == (int(want), True)
    # dot: x = trunc(a b / S) per step, underflow where a nonzero product truncates to 0
    p = a * b
    x = np.where(p < 0, -(-p // S), p // S)
    und = (p != 0) & (x == 0)
    wantd, evd = sfref.matmul_chain(bits, a[None, :], b[:, None])
    v, over, under = reduce_one(x, und, span, chunk, M)
    assert (v, over, under) == (int(wantd[0, 0]), bool(evd["overflow"][0, 0]), bool(evd["underflow"][0, 0]))
