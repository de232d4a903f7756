"""The scan and quantize kernels (sfb_scan / sfb_quantize) against the
oracle's float cast, bit for bit: codes, event counts and the L1 statistics,
for float32 and float64 input, one scale or one per row, strided rows."""
import numpy as np
import pytest

from conftest import golden
from oracle import sfref
from superfloat.python_b200 import _lib

pytestmark = pytest.mark.gpu


def stats_buf():
    import torch
    return torch.zeros(_lib.QSTATS_WORDS, dtype=torch.int64, device="cuda")


def run_quantize(vals, bits, scale=1.0, row_scale=None, ld_pad=0):
    import torch
    x = torch.as_tensor(vals)
    R, K = x.shape
    if ld_pad:
        big = torch.zeros(R, K + ld_pad, dtype=x.dtype)
        big[:, :K] = x
        xd = big.cuda()
    else:
        xd = x.cuda().contiguous()
    codes = torch.empty(R, K + 3, dtype=torch.int16, device="cuda")
    st = stats_buf()
    rs = None if row_scale is None else torch.as_tensor(row_scale, dtype=torch.float64).cuda()
    _lib.quantize(xd, R, K, xd.stride(0), scale, rs, bits, codes, K + 3, st)
    torch.cuda.synchronize()
    return codes[:, :K].cpu().numpy().astype(np.int64), _lib.qstats_view(st.cpu())


def check(vals, bits, scale=1.0, row_scale=None, ld_pad=0):
    v64 = np.asarray(vals).astype(np.float64)
    sc = scale if row_scale is None else np.asarray(row_scale, dtype=np.float64)[:, None]
    want, ev = sfref.cast_float(bits, v64, sc)
    got, q = run_quantize(vals, bits, scale, row_scale, ld_pad)
    np.testing.assert_array_equal(got, want)
    for e in ("overflow", "underflow", "invalid"):
        assert q[e] == int(ev[e].sum()), (bits, e)
    assert q["max_abs"] == int(np.abs(want).max(initial=0))
    assert q["max_row_l1"] == int(np.abs(want).sum(-1).max(initial=0))


def test_reference_cast_run():
    for c in golden("ref_runs.json")["cast"]:
        vals = np.array([[float(v) for v in c["values"]]])
        got, q = run_quantize(vals, c["bits"])
        assert got[0].tolist() == c["codes"]
        for e in ("overflow", "underflow", "invalid"):
            assert q[e] == sum(c[e]), (c["bits"], e)


@pytest.mark.parametrize("bits", [16, 13, 9, 8, 5, 4])
@pytest.mark.parametrize("dtype", ["float32", "float64"])
def test_random_rows_one_scale(bits, dtype, rng):
    S = 1 << (bits - 1)
    x = rng.normal(0, 1, (257, 300)) * rng.choice([1e-6, 1e-2, 1.0, 3.0], (257, 1))
    ties = (rng.integers(-S, S, (257, 20)) + 0.5) / S * 1.7
    x[:, :20] = ties                                    # exact ties of the scaled value
    x[5, 7] = np.nan
    x[9, 9] = np.inf
    x[10, 3] = -np.inf
    x = x.astype(dtype)
    check(x, bits, scale=1.7)


@pytest.mark.parametrize("bits", [16, 8])
def test_row_scales_and_strides(bits, rng):
    x = rng.normal(0, 1, (64, 129))
    rs = np.abs(x).max(1) / ((1 << (bits - 1)) - 1) * (1 << (bits - 1))
    rs[3] = 1.0
    x[3] = 0.0
    check(x, bits, row_scale=rs, ld_pad=5)
    check(x.astype(np.float32), bits, scale=0.25, ld_pad=3)


def test_shapes_empty_and_single():
    check(np.zeros((1, 1)), 16)
    check(np.array([[0.99998]]), 16)
    got, q = run_quantize(np.zeros((0, 4)), 16)
    assert got.shape == (0, 4) and q["max_abs"] == 0


def test_scan_counts_and_absmax(rng):
    import torch
    for dtype in (torch.float32, torch.float64):
        x = torch.tensor(rng.normal(0, 5, 1_000_003), dtype=dtype)
        x[17] = float("nan")
        x[18] = float("inf")
        x[19] = float("-inf")
        x[20] = float("nan")
        st = stats_buf()
        _lib.scan(x.cuda(), st)
        q = _lib.qstats_view(st.cpu())
        fin = torch.isfinite(x)
        assert q["nan"] == 2 and q["inf"] == 2
        assert q["absmax"] == float(x[fin].abs().max())
    st = stats_buf()
    _lib.scan(torch.zeros(5, device="cuda"), st)
    q = _lib.qstats_view(st.cpu())
    assert q["absmax"] == 0.0 and q["nan"] == 0


def test_argument_errors():
    import torch
    x = torch.zeros(4, 4, device="cuda")
    codes = torch.empty(4, 4, dtype=torch.int16, device="cuda")
    with pytest.raises(Exception):
        _lib.quantize(x, 4, 4, 4, 1.0, None, 17, codes, 4, stats_buf())
    with pytest.raises(Exception):
        _lib.quantize(x, 4, 4, 3, 1.0, None, 16, codes, 4, stats_buf())
    with pytest.raises(Exception):
        _lib.quantize(x, 4, 4, 4, 0.0, None, 16, codes, 4, stats_buf())
    with pytest.raises(TypeError):
        _lib.scan(torch.zeros(4, dtype=torch.int32, device="cuda"), stats_buf())
