"""Device I/O in the chip's sign-magnitude words: the conversion kernels over
every code and every 16-bit word, the elementwise ops reading and writing the
words inside the kernel, the host pipeline and the Device contract in that
format, all against the oracle."""
import numpy as np
import pytest
import torch

from oracle import sfref
from superfloat.python_b200 import FORMATS, _lib
from superfloat.python_b200._hostpath import HostPipeline

pytestmark = pytest.mark.gpu
ARITY = {"add": 2, "sub": 2, "mul": 2, "div": 2, "fma": 3, "neg": 1, "abs": 1, "sqrt": 1, "pow": 1}


@pytest.mark.parametrize("bits", [16, 12, 8, 5, 4])
def test_conversions_every_code_and_word(gpu, bits):
    M, _ = sfref.consts(bits)
    k = np.arange(-M, M + 1)
    codes = torch.from_numpy(k.astype(np.int16)).cuda()
    words = torch.empty_like(codes)
    _lib.to_bits(bits, codes, words)
    np.testing.assert_array_equal(words.cpu().numpy().view(np.uint16), sfref.to_bits(bits, k))
    allw = np.arange(1 << 16, dtype=np.uint16)
    wt = torch.from_numpy(allw.view(np.int16)).cuda()
    back = torch.empty_like(wt)
    cnt = torch.zeros(_lib.N_COUNTS, dtype=torch.int64, device="cuda")
    _lib.from_bits(bits, wt, back, cnt)
    want, fits = sfref.from_bits(bits, allw)
    ok = fits
    np.testing.assert_array_equal(back.cpu().numpy()[ok], want[ok])
    assert int(cnt[7]) == int((~fits).sum()) == (1 << 16) - (1 << bits)


@pytest.mark.parametrize("bits", [16, 9, 8, 4])
@pytest.mark.parametrize("op", list(ARITY))
def test_elementwise_on_words(gpu, op, bits, rng):
    M, _ = sfref.consts(bits)
    n = 50_003
    xs = [rng.integers(-M, M + 1, n) for _ in range(ARITY[op])]
    kw = {"n": 3} if op == "pow" else {}
    want, ev = sfref.ew(op, bits, *xs, **kw)
    words, masks = gpu.run_bits(op, FORMATS[bits], *(sfref.to_bits(bits, x) for x in xs), **kw)
    np.testing.assert_array_equal(words, sfref.to_bits(bits, want))
    for e, m in ev.items():
        np.testing.assert_array_equal(masks[e], m, err_msg=f"{op} sf{bits} {e}")


def test_negative_zero_and_bad_words(gpu):
    fmt = FORMATS[16]
    words, _ = gpu.run_bits("add", fmt, np.array([0x8000, 0x8001]), np.array([0x0001, 0x8000]))
    assert words.tolist() == [1, 0x8001]
    with pytest.raises(ValueError):
        gpu.run_bits("add", FORMATS[8], np.array([0x100]), np.array([1]))
    with pytest.raises(ValueError):
        gpu.upload_bits(FORMATS[8], np.array([3, 0x1FF]))


def test_reductions_in_word_format(gpu, rng):
    fmt = FORMATS[16]
    a = rng.integers(-3000, 3001, (5, 40))
    b = rng.integers(-32767, 32768, (40, 6))
    want, ev = sfref.matmul_chain(16, a, b)
    words, masks = gpu.run_bits("matmul", fmt, sfref.to_bits(16, a), sfref.to_bits(16, b))
    np.testing.assert_array_equal(words, sfref.to_bits(16, want))
    np.testing.assert_array_equal(masks["overflow"], ev["overflow"])
    s, sev = sfref.sum_chain(16, a, 1)
    words, masks = gpu.run_bits("sum", fmt, sfref.to_bits(16, a), axis=1)
    np.testing.assert_array_equal(words, sfref.to_bits(16, s))


def test_host_pipeline_in_word_format(gpu, rng):
    pipe = HostPipeline(gpu, chunk=1 << 12)
    n = 3 * (1 << 12) + 5
    x, y = rng.integers(-32767, 32768, n), rng.integers(-32767, 32768, n)
    hs = []
    for v in (x, y):
        t = torch.empty(n, dtype=torch.int16, pin_memory=True)
        t.copy_(torch.from_numpy(sfref.to_bits(16, v).view(np.int16)))
        hs.append(t)
    out = torch.empty(n, dtype=torch.int16, pin_memory=True)
    counts = pipe.run("mul", FORMATS[16], *hs, out=out, layout="signmag")
    want, ev = sfref.mul(16, x, y)
    np.testing.assert_array_equal(out.numpy().view(np.uint16), sfref.to_bits(16, want))
    assert int(counts[1]) == int(ev["underflow"].sum())
