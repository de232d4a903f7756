"""Elementwise kernels vs the oracle, through the C ABI (B200Device), bit for bit:
codes, per-output event masks and event counts."""
import hashlib

import numpy as np
import pytest

from conftest import golden
from oracle import sfref
from superfloat.python_b200 import FORMATS, workloads

pytestmark = pytest.mark.gpu

OPS = ["add", "sub", "mul", "div", "fma", "neg", "abs", "sqrt", "pow"]
ARITY = {"add": 2, "sub": 2, "mul": 2, "div": 2, "fma": 3, "neg": 1, "abs": 1, "sqrt": 1, "pow": 1}


def sha_codes(c):
    return hashlib.sha256(np.ascontiguousarray(c, dtype="<i2").tobytes()).hexdigest()


def sha_mask(m):
    return hashlib.sha256(np.packbits(np.asarray(m, bool).ravel()).tobytes()).hexdigest()


def edge_codes(bits, n, rng):
    """Random codes with every edge value mixed in: 0, +-1, +-M, +-(M-1), +-S/2."""
    M = (1 << (bits - 1)) - 1
    x = rng.integers(-M, M + 1, n)
    edges = np.array([0, 1, -1, M, -M, M - 1, -(M - 1), (M + 1) // 2, -((M + 1) // 2), 2, -2])
    idx = rng.integers(0, n, n // 4)
    x[idx] = rng.choice(edges, idx.size)
    small = rng.integers(0, n, n // 8)
    x[small] = rng.integers(-min(M, 200), min(M, 200) + 1, small.size)
    return x


def check_against_oracle(gpu, op, bits, xs, **kw):
    fmt = FORMATS[bits]
    want, ev = sfref.ew(op, bits, *xs, **kw)
    got, masks = gpu.run(op, fmt, *xs, **kw)
    np.testing.assert_array_equal(got, want)
    assert set(masks) == set(ev), (op, set(masks), set(ev))
    for e, m in ev.items():
        np.testing.assert_array_equal(masks[e], m, err_msg=f"{op} sf{bits} {e}")
    # counts from the device equal the oracle's mask counts
    import torch
    ts = [gpu.upload(x) for x in xs]
    _, cnt, _ = gpu.run_device(op, fmt, *ts, **kw)
    cnt = cnt.cpu().numpy()
    names = ["overflow", "underflow", "divide", "invalid"]
    for i, e in enumerate(names):
        assert int(cnt[i]) == int(np.count_nonzero(ev.get(e, False))), (op, bits, e)
    torch.cuda.synchronize()


@pytest.mark.parametrize("bits", [16, 15, 12, 9, 8, 5, 4])
@pytest.mark.parametrize("op", OPS)
def test_random_and_edges(gpu, op, bits, rng):
    n = 100_003                       # not a multiple of 8: vector body plus a scalar tail
    xs = [edge_codes(bits, n, rng) for _ in range(ARITY[op])]
    kw = {"n": int(rng.integers(2, 6))} if op == "pow" else {}
    check_against_oracle(gpu, op, bits, xs, **kw)


@pytest.mark.parametrize("op", ["add", "div", "fma"])
def test_broadcast_and_small_shapes(gpu, op, rng):
    M = 32767
    shapes = [((3, 5), (5,)), ((1,), (7, 1)), ((), (4, 4)), ((2, 1, 3), (1, 4, 1))]
    for sa, sb in shapes:
        a = rng.integers(-M, M + 1, sa)
        b = rng.integers(-M, M + 1, sb)
        xs = [a, b] + ([rng.integers(-M, M + 1, sb)] if op == "fma" else [])
        check_against_oracle(gpu, op, 16, xs)


def test_every_length_and_misaligned_views(gpu, rng):
    """Lengths 1..40 and views starting off the 16-byte boundary take the scalar path."""
    import torch
    fmt = FORMATS[16]
    for n in list(range(1, 41)) + [1023, 1025]:
        a = rng.integers(-32767, 32768, n)
        b = rng.integers(-32767, 32768, n)
        check_against_oracle(gpu, "add", 16, [a, b])
    a = rng.integers(-32767, 32768, 4097)
    b = rng.integers(-32767, 32768, 4097)
    ta, tb = gpu.upload(a), gpu.upload(b)
    o, cnt, fl = gpu.run_device("mul", fmt, ta[1:], tb[1:], flags=True)
    want, ev = sfref.mul(16, a[1:], b[1:])
    np.testing.assert_array_equal(o.cpu().numpy(), want)
    np.testing.assert_array_equal((fl.cpu().numpy() & 2) != 0, ev["underflow"])
    assert int(cnt[1]) == int(ev["underflow"].sum())
    torch.cuda.synchronize()


def test_golden_vectors_on_device(gpu):
    cases = golden("elementwise.json")["cases"]
    groups = {}
    for c in cases:
        groups.setdefault((c["op"], c["bits"]), []).append(c)
    bit = {"overflow": 1, "underflow": 2, "divide": 4, "invalid": 8}
    for (op, bits), cs in groups.items():
        xs = [np.array([c["in"][i] for c in cs]) for i in range(ARITY[op])]
        got, masks = gpu.run(op, FORMATS[bits], *xs)
        assert got.tolist() == [c["out"] for c in cs], (op, bits)
        for j, c in enumerate(cs):
            hit = [e for e, m in masks.items() if m[j]]
            assert hit == ([c["event"]] if c["event"] else []), (op, bits, c)
    assert sum(len(v) for v in groups.values()) == len(cases)


def test_workload_2_20_matches_reference_run(gpu):
    runs = golden("ref_runs.json")["elementwise"]
    x, y, z, d = workloads.elementwise(1 << 20, 0)
    args = {"add": (x, y), "sub": (x, y), "mul": (x, y), "fma": (x, y, z), "div": (x, d)}
    for op, r in runs.items():
        got, masks = gpu.run(op, FORMATS[16], *args[op])
        assert sha_codes(got) == r["codes"], op
        for e, m in masks.items():
            assert int(m.sum()) == r[f"n_{e}"] and sha_mask(m) == r[f"mask_{e}"], (op, e)


def test_workload_full_size_2_26(gpu):
    """The 2^26-element workload: full-size event counts against the oracle's,
    and a random sample of 2^18 outputs element by element."""
    import torch
    n = 1 << 26
    x, y, z, d = workloads.elementwise(n, 0)
    tx, ty, tz, td = (gpu.upload(v) for v in (x, y, z, d))
    fmt = FORMATS[16]
    sample = np.random.default_rng(5).integers(0, n, 1 << 18)
    for op, args, targs in (("add", (x, y), (tx, ty)), ("sub", (x, y), (tx, ty)), ("mul", (x, y), (tx, ty)),
                            ("fma", (x, y, z), (tx, ty, tz)), ("div", (x, d), (tx, td))):
        o, cnt, fl = gpu.run_device(op, fmt, *targs, flags=True)
        o = o.cpu().numpy()
        fl = fl.cpu().numpy()
        want, ev = sfref.ew(op, 16, *(a[sample] for a in args))
        np.testing.assert_array_equal(o[sample], want, err_msg=op)
        for e, m in ev.items():
            b = {"overflow": 1, "underflow": 2, "divide": 4}[e]
            np.testing.assert_array_equal((fl[sample] & b) != 0, m, err_msg=f"{op} {e}")
        cnt = cnt.cpu().numpy()
        if op == "div":
            zero = d == 0
            over = ~zero & (x != 0) & (np.abs(x) >= np.abs(d))
            assert int(cnt[2]) == int(zero.sum()) and int(cnt[0]) == int(over.sum())
        else:
            _, evf = sfref.ew(op, 16, *args)
            for i, e in enumerate(("overflow", "underflow")):
                assert int(cnt[i]) == int(np.count_nonzero(evf.get(e, False))), (op, e)
        assert int((fl != 0).sum()) <= n
    torch.cuda.synchronize()


def test_host_pipeline_and_plugin_contract(gpu, rng):
    """Host-resident codes through the chunked two-stream pipeline, and the
    int64 Device.run contract through the pooled stager (small chunks, so
    several chunks reuse each slot), equal the oracle."""
    import torch
    from superfloat.python_b200._device import _EVENT_BIT, OP_EVENTS
    from superfloat.python_b200._hostpath import HostPipeline, PluginStager
    pipe = HostPipeline(gpu, chunk=1 << 12)
    stager = PluginStager(gpu, chunk=1 << 12)
    n = 3 * (1 << 12) + 77
    for op in ("add", "mul", "div", "fma", "sqrt"):
        xs = [edge_codes(16, n, rng) for _ in range(ARITY[op])]
        hs = []
        for v in xs:
            t = torch.empty(n, dtype=torch.int16, pin_memory=True)
            t.copy_(torch.from_numpy(v))
            hs.append(t)
        out = torch.empty(n, dtype=torch.int16, pin_memory=True)
        fl = torch.empty(n, dtype=torch.uint8, pin_memory=True)
        counts = pipe.run(op, FORMATS[16], *hs, out=out, flags_out=fl)
        want, ev = sfref.ew(op, 16, *xs)
        np.testing.assert_array_equal(out.numpy(), want)
        for i, e in enumerate(("overflow", "underflow", "divide", "invalid")):
            assert int(counts[i]) == int(np.count_nonzero(ev.get(e, False))), (op, e)
        for _ in range(2):                                  # the second call reuses the staging buffers
            codes, masks, cnt = stager.run(op, 16, [np.ascontiguousarray(x, dtype=np.int64) for x in xs],
                                           OP_EVENTS[op], _EVENT_BIT)
            np.testing.assert_array_equal(codes, want)
            assert set(masks) == set(ev)
            for e, m in ev.items():
                np.testing.assert_array_equal(masks[e], m)
            np.testing.assert_array_equal(cnt, counts)


def test_device_run_stages_large_calls(gpu):
    """Device.run on 2^20 + 5 codes (the staged path) and with a broadcast
    operand (the direct path) equals the oracle, codes and masks."""
    from superfloat.python_b200._device import STAGED_MIN_ELEMENTS
    rng = np.random.default_rng(3)
    n = STAGED_MIN_ELEMENTS + 5
    a = rng.integers(-32767, 32768, n)
    b = rng.integers(-32767, 32768, n)
    b[::101] = 0
    for op, xs in (("div", (a, b)), ("add", (a, b)), ("mul", (a, b[:1]))):
        got, masks = gpu.run(op, FORMATS[16], *xs)
        want, ev = sfref.ew(op, 16, *xs)
        np.testing.assert_array_equal(got, want)
        for e, m in ev.items():
            np.testing.assert_array_equal(masks[e], np.broadcast_to(m, got.shape))
    assert gpu._stager is not None


def test_multi_op_pipeline_equals_the_oracle(gpu, rng):
    """Several ops over shared host operands, each operand copied in once per
    chunk (small chunks: several per call, both streams): every result and
    every op's counts equal the oracle, twice in a row."""
    import torch
    from superfloat.python_b200._hostpath import MultiOpPipeline
    n = 5 * (1 << 12) + 3
    vals = {nm: edge_codes(16, n, rng) for nm in ("x", "y", "z")}
    ops = [("add", ("x", "y")), ("div", ("y", "x")), ("fma", ("x", "y", "z")), ("neg", ("z",)), ("mul", ("z", "x"))]
    pipe = MultiOpPipeline(gpu, ("x", "y", "z"), ops, chunk=1 << 12)
    hin = {}
    for nm, v in vals.items():
        t = torch.empty(n, dtype=torch.int16, pin_memory=True)
        t.copy_(torch.from_numpy(v))
        hin[nm] = t
    def check(outs, counts):
        for i, (op, args) in enumerate(ops):
            want, ev = sfref.ew(op, 16, *(vals[a] for a in args))
            np.testing.assert_array_equal(outs[i].numpy(), want, err_msg=op)
            for j, e in enumerate(("overflow", "underflow", "divide", "invalid")):
                assert int(counts[i][j]) == int(np.count_nonzero(ev.get(e, False))), (op, e)

    for _ in range(2):
        outs = [torch.empty(n, dtype=torch.int16, pin_memory=True) for _ in ops]
        check(outs, pipe.run(FORMATS[16], hin, outs))
    # two calls queued before either is read
    outs1 = [torch.empty(n, dtype=torch.int16, pin_memory=True) for _ in ops]
    outs2 = [torch.empty(n, dtype=torch.int16, pin_memory=True) for _ in ops]
    p1 = pipe.run_async(FORMATS[16], hin, outs1)
    p2 = pipe.run_async(FORMATS[16], hin, outs2)
    check(outs1, p1.result())
    check(outs2, p2.result())
