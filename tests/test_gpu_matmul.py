"""Chain and wide matmul kernels vs the oracle through the C ABI, bit for bit."""
import hashlib

import numpy as np
import pytest

from conftest import golden
from oracle import native, sfref
from superfloat.python_b200 import FORMATS, workloads

pytestmark = pytest.mark.gpu


def sha_codes(c):
    return hashlib.sha256(np.ascontiguousarray(c, dtype="<i2").tobytes()).hexdigest()


def sha_mask(m):
    return hashlib.sha256(np.packbits(np.asarray(m, bool).ravel()).tobytes()).hexdigest()


SHAPES = [(1, 1, 1), (1, 7, 1), (5, 3, 9), (64, 64, 32), (65, 63, 33), (130, 70, 257), (3, 200, 64),
          (100, 1, 100), (7, 7, 0), (5, 9, 4099), (64, 64, 1000)]


def _codes(rng, bits, shape, frac=1.0):
    M = (1 << (bits - 1)) - 1
    lim = max(1, int(M * frac))
    return rng.integers(-lim, lim + 1, shape)


@pytest.mark.parametrize("bits", [16, 13, 8, 4])
@pytest.mark.parametrize("frac", [1.0, 0.02])
def test_chain_random_shapes(gpu, bits, frac, rng):
    for (M, N, K) in SHAPES:
        A = _codes(rng, bits, (M, K), frac)
        B = _codes(rng, bits, (K, N))
        want, ev = sfref.matmul_chain(bits, A, B)
        got, masks = gpu.run("matmul", FORMATS[bits], A, B)
        np.testing.assert_array_equal(got, want, err_msg=f"{M}x{N}x{K}")
        np.testing.assert_array_equal(masks["overflow"], ev["overflow"])
        np.testing.assert_array_equal(masks["underflow"], ev["underflow"])


def _chain_small_tier(M, N, sms):
    """Which tiling the general chain picks for a 2-D problem too small for
    32 x 64 tiles (sfb_chain.cu launch_chain): 32x32, 16x32 or 8x32; None above."""
    c = lambda rows, cols: -(-M // rows) * -(-N // cols)
    if c(32, 64) >= sms:
        return None
    if c(32, 32) >= sms:
        return "32x32"
    return "16x32" if c(16, 32) >= sms // 2 else "8x32"


@pytest.mark.parametrize("bits", [16, 8])
def test_chain_small_problem_tilings(gpu, bits, rng):
    """Every tiling of the small-problem tier, on ragged shapes with odd K
    (scalar loads) and even K (vector loads), against the oracle."""
    import torch
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    shapes = [(400, 390, 97), (448, 352, 64), (300, 200, 333), (280, 256, 96), (100, 90, 77), (24, 40, 128)]
    tiers = set()
    for (M, N, K) in shapes:
        tiers.add(_chain_small_tier(M, N, sms))
        A = _codes(rng, bits, (M, K))
        B = _codes(rng, bits, (K, N))
        A[0] = _codes(rng, bits, K, 0.01)
        want, ev = sfref.matmul_chain(bits, A, B)
        got, masks = gpu.run("matmul", FORMATS[bits], A, B)
        np.testing.assert_array_equal(got, want, err_msg=f"{M}x{N}x{K}")
        np.testing.assert_array_equal(masks["overflow"], ev["overflow"])
        np.testing.assert_array_equal(masks["underflow"], ev["underflow"])
    if sms == 148:
        assert tiers == {"32x32", "16x32", "8x32"}


def test_chain_golden_dot(gpu):
    for c in golden("chain.json")["cases"]:
        if c["op"] != "dot":
            continue
        a, b = np.array(c["in"][0]), np.array(c["in"][1])
        got, masks = gpu.run("matmul", FORMATS[c["bits"]], a[None, :], b[:, None])
        assert int(got[0, 0]) == c["out"]
        assert {e for e in masks if masks[e][0, 0]} == set(c["events"])


def test_chain_reference_runs(gpu):
    for c in golden("ref_runs.json")["small_chain"]:
        got, masks = gpu.run("matmul", FORMATS[c["bits"]], np.array(c["a"]), np.array(c["b"]))
        assert got.tolist() == c["out"]
        assert masks["overflow"].astype(int).tolist() == c["overflow"]
        assert masks["underflow"].astype(int).tolist() == c["underflow"]


def test_chain_512_workload(gpu):
    A, B = workloads.chain_square(512, 0)
    got, masks = gpu.run("matmul", FORMATS[16], A, B)
    r = golden("ref_runs.json")["chain_512"]
    assert sha_codes(got) == r["codes"]
    assert sha_mask(masks["overflow"]) == r["overflow"] and sha_mask(masks["underflow"]) == r["underflow"]


def test_chain_batched_and_broadcast(gpu, rng):
    A = _codes(rng, 16, (2, 3, 17, 40), 0.05)
    B = _codes(rng, 16, (40, 9))
    for a, b in ((A, B), (A[0, 0], _codes(rng, 16, (2, 3, 40, 9))), (A, _codes(rng, 16, (3, 40, 9)))):
        want, ev = sfref.matmul_chain(16, a, b)
        got, masks = gpu.run("matmul", FORMATS[16], a, b)
        np.testing.assert_array_equal(got, want)
        np.testing.assert_array_equal(masks["overflow"], ev["overflow"])
        np.testing.assert_array_equal(masks["underflow"], ev["underflow"])


def test_chain_fused_bias(gpu, rng):
    """matmul then one saturating add of a bias row; overflow is the union."""
    import torch
    fmt = FORMATS[16]
    A = _codes(rng, 16, (77, 300), 0.1)
    B = _codes(rng, 16, (300, 50))
    bias = _codes(rng, 16, (50,))
    q, ev = sfref.matmul_chain(16, A, B)
    y, ev2 = sfref.add(16, q, bias[None, :])
    o, cnt, fl = gpu.run_device("matmul", fmt, gpu.upload(A), gpu.upload(B), flags=True, bias=gpu.upload(bias))
    np.testing.assert_array_equal(o.cpu().numpy(), y)
    fl = fl.cpu().numpy()
    over = ev["overflow"] | ev2["overflow"]
    np.testing.assert_array_equal((fl & 1) != 0, over)
    np.testing.assert_array_equal((fl & 2) != 0, ev["underflow"])
    assert int(cnt[0]) == int(over.sum()) and int(cnt[1]) == int(ev["underflow"].sum())
    torch.cuda.synchronize()


# --- wide ----------------------------------------------------------------------------------

@pytest.mark.parametrize("mx", ["v4.9.2", "v4.8.1"])
def test_wide_mxref_golden(gpu, mx):
    from superfloat.python_b200 import B200Device
    dev = B200Device(0, mx=mx, name=f"b200-{mx}")
    for c in golden("wide_mx.json")["cases"]:
        if c["mx"] != mx:
            continue
        got, _ = dev.run("matmul_wide", FORMATS[c["bits"]], np.array(c["a"]), np.array(c["b"]), shift=c["shift"])
        assert got.tolist() == c["out"], (c["bits"], c["shift"])


def test_wide_shift_arrays_golden(gpu):
    for c in golden("wide_shift.json")["cases"]:
        sh = c["shift"] if isinstance(c["shift"], int) else np.array(c["shift"])
        got, masks = gpu.run("matmul_wide", FORMATS[c["bits"]], np.array(c["a"]), np.array(c["b"]), shift=sh,
                             mx=c["target"])
        assert got.tolist() == c["out"]
        assert masks["overflow"].astype(int).tolist() == c["overflow"]
        assert masks["underflow"].astype(int).tolist() == c["underflow"]


def test_wide_reference_runs(gpu):
    for c in golden("ref_runs.json")["small_wide"]:
        got, masks = gpu.run("matmul_wide", FORMATS[c["bits"]], np.array(c["a"]), np.array(c["b"]),
                             shift=c["shift"], mx=c["mx"])
        assert got.tolist() == c["out"]
        assert masks["overflow"].astype(int).tolist() == c["overflow"]
        assert masks["underflow"].astype(int).tolist() == c["underflow"]


@pytest.mark.parametrize("bits", [16, 12, 9, 8, 4])
@pytest.mark.parametrize("mx", ["v4.9.2", "v4.8.1"])
def test_wide_random_shapes(gpu, bits, mx, rng):
    for (M, N, K) in SHAPES:
        A = _codes(rng, bits, (M, K))
        B = _codes(rng, bits, (K, N))
        shift = int(rng.integers(-8, 9))
        want, ev = sfref.matmul_wide(bits, A, B, shift, mx, acc_fn=native.wide_acc)
        got, masks = gpu.run("matmul_wide", FORMATS[bits], A, B, shift=shift, mx=mx)
        np.testing.assert_array_equal(got, want, err_msg=f"{M}x{N}x{K} sf{bits} {mx}")
        np.testing.assert_array_equal(masks["overflow"], ev["overflow"])
        np.testing.assert_array_equal(masks["underflow"], ev["underflow"])


def test_wide_accumulator_clips(gpu, rng):
    """Large K with same-sign operands drives the accumulator into its limit."""
    for bits, mx in ((16, "v4.9.2"), (16, "v4.8.1"), (8, "v4.8.1")):
        M_ = (1 << (bits - 1)) - 1
        A = rng.integers(M_ // 2, M_ + 1, (9, 4000))
        B = rng.integers(M_ // 2, M_ + 1, (4000, 5)) * rng.choice([-1, 1], (1, 5))
        want, ev = sfref.matmul_wide(bits, A, B, 0, mx, acc_fn=native.wide_acc)
        got, masks = gpu.run("matmul_wide", FORMATS[bits], A, B, shift=0, mx=mx)
        np.testing.assert_array_equal(got, want)
        np.testing.assert_array_equal(masks["overflow"], ev["overflow"])
        if mx == "v4.8.1":
            assert ev["overflow"].any()


def test_wide_8192_workload_first_rows(gpu):
    """The 8192^3 wide workload on the GPU; rows 0..511 against the reference's run."""
    import torch
    A, B = workloads.wide_square(8192, 8192, 8192, 0)
    o, cnt, fl = gpu.run_device("matmul_wide", FORMATS[16], gpu.upload(A), gpu.upload(B), flags=True, shift=0)
    r = golden("ref_runs.json")["wide_8192_rows16"]
    o16 = o[:16].cpu().numpy()
    f16 = fl[:16].cpu().numpy()
    assert sha_codes(o16) == r["codes"]
    assert sha_mask((f16 & 1) != 0) == r["overflow"] and sha_mask((f16 & 2) != 0) == r["underflow"]
    # rows 0..511 in blocks of 16 against the reference's own compiled MX loop
    wr = golden("wide_8192_rows512.json")
    o512, f512 = o[:wr["rows"]].cpu().numpy(), fl[:wr["rows"]].cpu().numpy()
    for b in wr["blocks"]:
        r0, r1 = b["r0"], b["r0"] + wr["block"]
        assert sha_codes(o512[r0:r1]) == b["codes"], r0
        assert sha_mask((f512[r0:r1] & 1) != 0) == b["overflow"], r0
        assert sha_mask((f512[r0:r1] & 2) != 0) == b["underflow"], r0
    cnt = cnt.cpu().numpy()
    frac = cnt[0] / (8192 * 8192)
    assert 0.005 < frac < 0.02 and cnt[4] == 0       # ~1% saturate, no accumulator clip
    # a few more rows against the C oracle
    rows = np.array([17, 4095, 8191])
    want, ev = sfref.matmul_wide(16, A[rows], B, 0, acc_fn=native.wide_acc)
    np.testing.assert_array_equal(o[rows].cpu().numpy(), want)
    torch.cuda.synchronize()
