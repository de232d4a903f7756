"""The wide matmul's tensor-core path (tcgen05 int8 passes + bit-sliced
remainder) against the oracle, bit for bit: ragged shapes, the SF16-block
widths, shift arrays, batches, and outputs the clip bound does not prove safe
(recomputed exactly on the CUDA cores)."""
import numpy as np
import pytest

from oracle import native, sfref
from superfloat.python_b200 import FORMATS, _lib

pytestmark = pytest.mark.gpu


def _run(gpu, bits, A, B, shift=0, flags=True):
    import torch
    o, cnt, fl = gpu.run_device("matmul_wide", FORMATS[bits], gpu.upload(A), gpu.upload(B), flags=flags,
                                shift=shift)
    c = cnt.cpu().numpy()
    _lib.check_counts(c)
    torch.cuda.synchronize()
    return o.cpu().numpy(), c, (None if fl is None else fl.cpu().numpy())


def _want(bits, A, B, shift):
    return sfref.matmul_wide(bits, A, B, shift, acc_fn=native.wide_acc)


def test_path_is_taken_for_large_problems(gpu):
    assert _lib.wide_workspace(16, "v4.9.2", 1, 300, 260, 1000) > 0      # tensor-core path
    assert _lib.wide_workspace(16, "v4.8.1", 1, 300, 260, 1000) == 0     # CUDA-core path
    assert _lib.wide_workspace(8, "v4.9.2", 1, 300, 260, 1000) == 0      # SF8 block
    assert _lib.wide_workspace(16, "v4.9.2", 1, 8, 8, 8) == 0            # too small to pay


@pytest.mark.parametrize("bits", [16, 14, 12, 9])
def test_ragged_random(gpu, bits):
    rng = np.random.default_rng(bits)
    M_ = (1 << (bits - 1)) - 1
    for (M, N, K) in ((300, 260, 1000), (128, 128, 256), (129, 257, 130)):
        A = rng.integers(-M_, M_ + 1, (M, K)) // rng.integers(1, 60)
        B = rng.integers(-M_, M_ + 1, (K, N))
        shift = int(rng.integers(-4, 5))
        got, cnt, fl = _run(gpu, bits, A, B, shift)
        want, ev = _want(bits, A, B, shift)
        np.testing.assert_array_equal(got, want, err_msg=f"sf{bits} {M}x{N}x{K}")
        np.testing.assert_array_equal((fl & 1) != 0, ev["overflow"])
        np.testing.assert_array_equal((fl & 2) != 0, ev["underflow"])
        assert int(cnt[0]) == int(ev["overflow"].sum()) and int(cnt[1]) == int(ev["underflow"].sum())


def test_edge_codes_and_zero_rows(gpu):
    rng = np.random.default_rng(7)
    M, N, K = 200, 140, 600
    A = rng.choice(np.array([0, 1, -1, 63, -64, 255, -256, 32767, -32767, 16384, 12345]), (M, K))
    B = rng.choice(np.array([0, 1, -1, 64, -63, 256, -255, 32767, -32767, 8191]), (K, N))
    A[5] = 0
    B[:, 7] = 0
    A = A // 64                                  # keep most outputs below the clip bound
    got, _, _ = _run(gpu, 16, A, B, -3)
    want, _ = _want(16, A, B, -3)
    np.testing.assert_array_equal(got, want)


def test_shift_arrays(gpu):
    rng = np.random.default_rng(11)
    M, N, K = 256, 192, 512
    A = rng.integers(-4000, 4001, (M, K))
    B = rng.integers(-32767, 32768, (K, N))
    for sh in (rng.integers(-8, 4, (M, 1)), rng.integers(-8, 4, (N,)), rng.integers(-32, 32, (M, N))):
        got, _, _ = _run(gpu, 16, A, B, sh)
        want, _ = _want(16, A, B, sh)
        np.testing.assert_array_equal(got, want)


def test_outputs_beyond_the_clip_bound_are_exact(gpu):
    """Full-range codes with K = 4096 are not proven clip-free: recomputed
    exactly on the CUDA cores; same-sign operands clip for real."""
    rng = np.random.default_rng(5)
    M, N, K = 128, 128, 4096
    A = rng.integers(-32767, 32768, (M, K))
    B = rng.integers(-32767, 32768, (K, N))
    A[:4] = np.abs(A[:4])
    B[:, :4] = np.abs(B[:, :4])
    got, cnt, fl = _run(gpu, 16, A, B, -12)
    want, ev = _want(16, A, B, -12)
    np.testing.assert_array_equal(got, want)
    np.testing.assert_array_equal((fl & 1) != 0, ev["overflow"])
    acc, clip, _ = native.wide_acc(16, A, B)
    np.testing.assert_array_equal((fl & 16) != 0, clip)
    assert clip[:4, :4].all() and int(cnt[4]) == int(clip.sum())


def test_batched(gpu):
    rng = np.random.default_rng(9)
    A = rng.integers(-2000, 2001, (3, 130, 300))
    B = rng.integers(-32767, 32768, (300, 140))
    got, _, _ = _run(gpu, 16, A, B, -1)
    want, _ = _want(16, A.reshape(-1, 300), B, -1)
    np.testing.assert_array_equal(got.reshape(-1, 140), want)


def test_a_wait_that_runs_out_is_reported_and_the_next_call_is_exact(gpu):
    """Failure detection without a fault: with a 64-poll limit and the MMA
    thread first waiting on a barrier nothing arrives on, every CTA of the
    GEMM gives up, lets its copies in flight land, frees its tensor memory and
    counts the failure; the host raises SFDeviceError from that count, and the
    next call on the same context (default limit) is bit-exact."""
    from superfloat.python_b200._errors import SFDeviceError
    lib = _lib.load()
    rng = np.random.default_rng(21)
    A = rng.integers(-3000, 3001, (300, 1000))
    B = rng.integers(-32767, 32768, (1000, 260))
    try:
        assert lib.sfb_wide_wait_limit(64, 1) == _lib.SFB_OK
        with pytest.raises(SFDeviceError, match="gave up waiting"):
            _run(gpu, 16, A, B, -1)
    finally:
        lib.sfb_wide_wait_limit(0, 0)
    got, cnt, fl = _run(gpu, 16, A, B, -1)
    want, ev = _want(16, A, B, -1)
    np.testing.assert_array_equal(got, want)
    np.testing.assert_array_equal((fl & 1) != 0, ev["overflow"])
    assert int(cnt[5]) == 0


def test_prepared_b_equals_the_plain_call(gpu):
    """B prepared once (sfb_wide_prepare_b) and used by calls with different
    A (ragged, batched, shift arrays) gives the plain call's codes, flags and
    counts; a width with no prepared form (sf8) falls back to B's codes."""
    import torch
    dev = torch.device("cuda", 0)
    rng = np.random.default_rng(31)
    K, N = 700, 300
    B = rng.integers(-32767, 32768, (K, N))
    tB = torch.from_numpy(B).to(torch.int16).to(dev)
    nbytes = _lib.wide_prepared_b_bytes(16, "v4.9.2", N, K)
    assert nbytes > 0 and _lib.wide_prepared_b_bytes(8, "v4.9.2", N, K) == 0
    prep = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    _lib.wide_prepare_b(16, "v4.9.2", tB, N, K, N, prep)
    for batch, M, shift in ((1, 257, -2), (3, 130, 0), (1, 400, rng.integers(-6, 3, (400, N)))):
        A = rng.integers(-3000, 3001, (batch, M, K))
        tA = torch.from_numpy(A).to(torch.int16).to(dev)
        ws = torch.empty(max(1, _lib.wide_workspace(16, "v4.9.2", batch, M, N, K)), dtype=torch.uint8, device=dev)
        sh_t = None if np.isscalar(shift) else torch.from_numpy(np.asarray(shift)).to(torch.int8).to(dev)
        sh = 0 if sh_t is not None else int(shift)
        ss = (0, N, 1) if sh_t is not None else (0, 0, 0)
        res = []
        for use_prep in (False, True):
            out = torch.empty(batch, M, N, dtype=torch.int16, device=dev)
            fl = torch.empty(batch, M, N, dtype=torch.uint8, device=dev)
            cnt = torch.zeros(8, dtype=torch.int64, device=dev)
            if use_prep:
                _lib.matmul_wide_prepared(16, "v4.9.2", tA, tB, prep, sh_t, sh, out, fl, cnt, batch, M, N, K, K, N,
                                          M * K, M * N, *ss, ws)
            else:
                _lib.matmul_wide(16, "v4.9.2", tA, tB, sh_t, sh, out, fl, cnt, batch, M, N, K, K, N, M * K, 0, M * N,
                                 *ss, ws)
            torch.cuda.synchronize()
            res.append((out.cpu().numpy(), fl.cpu().numpy(), cnt.cpu().numpy()))
        for x, y in zip(*res):
            np.testing.assert_array_equal(x, y)
        want, _ = _want(16, A[0], B, shift)
        np.testing.assert_array_equal(res[1][0][0], want)
        assert int(res[1][2][5]) == 0
    # sf8 has no prepared form: prep NULL reads B's codes
    A8 = rng.integers(-127, 128, (200, K))
    B8 = rng.integers(-127, 128, (K, N))
    tA8 = torch.from_numpy(A8).to(torch.int16).to(dev)
    tB8 = torch.from_numpy(B8).to(torch.int16).to(dev)
    out = torch.empty(200, N, dtype=torch.int16, device=dev)
    cnt = torch.zeros(8, dtype=torch.int64, device=dev)
    _lib.matmul_wide_prepared(8, "v4.9.2", tA8, tB8, None, None, -1, out, None, cnt, 1, 200, N, K, K, N, 0, 200 * N,
                              0, 0, 0, None)
    want, _ = sfref.matmul_wide(8, A8, B8, -1)
    np.testing.assert_array_equal(out.cpu().numpy(), want)
