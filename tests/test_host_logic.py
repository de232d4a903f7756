"""Host-side logic of the runtime, no GPU: casts, pre-flight verdicts, error
policy, config and accumulation-mode scoping, dtype resolution."""
import asyncio
import warnings

import numpy as np
import pytest

from conftest import golden
import superfloat.python_b200 as sf
from superfloat.python_b200 import _preflight
from superfloat.python_b200._cast import cast_array
from superfloat.python_b200._format import FORMATS


def test_cast_matches_reference():
    for c in golden("ref_runs.json")["cast"]:
        vals = np.array([float(v) for v in c["values"]])
        k, ev = cast_array(FORMATS[c["bits"]], vals)
        assert k.tolist() == c["codes"]
        for e in ("overflow", "underflow", "invalid"):
            assert ev[e].astype(int).tolist() == c[e], (c["bits"], e)


def test_cast_integers_and_bools():
    f = FORMATS[16]
    k, ev = cast_array(f, np.array([0, 3, -2]))
    assert k.tolist() == [0, 32767, -32767] and ev["overflow"].tolist() == [False, True, True]
    k, _ = cast_array(f, np.array([True, False]))
    assert k.tolist() == [32767, 0]


def test_host_array_construction_and_policy():
    x = sf.asarray([0.5, -0.25, 0.0], dtype=sf.sf16)
    assert x.codes.tolist() == [16384, -8192, 0] and x.device == "host" and x.status is None
    with pytest.raises(sf.SFOverflowError):
        sf.asarray([1.0], dtype=sf.sf16)
    with sf.errstate(over="ignore"):
        assert sf.asarray([1.0], dtype=sf.sf16).codes.tolist() == [32767]
    with pytest.raises(sf.SFInvalidError):
        sf.asarray([np.nan], dtype=sf.sf8)
    with pytest.warns(sf.SFUnderflowWarning):
        sf.asarray([1e-9], dtype=sf.sf16)
    with pytest.raises(sf.SFTypeError):
        sf.asarray([0.5])
    with pytest.raises(sf.SFInvalidError):
        sf.from_codes(np.array([40000]), sf.sf16)
    assert sf.from_codes(np.array([5, -7]), "sf8").codes.tolist() == [5, -7]
    assert sf.dtype(12) is sf.sf12 and sf.dtype("sf4") is sf.sf4 and sf.sf16.bits == 16
    assert x.bits.tolist() == [16384, 32768 | 8192, 0]
    assert x.numpy().tolist() == [0.5, -0.25, 0.0]


def test_preflight_verdicts():
    f = FORMATS[16]
    M = f.max_code
    assert _preflight.check("add", f, np.array([100]), np.array([200])).kind == "safe"
    assert _preflight.check("add", f, np.array([30000, 29000]), np.array([20000, 21000])).kind == "certain"
    assert _preflight.check("sub", f, np.array([30000]), np.array([-20000])).kind == "certain"
    assert _preflight.check("add", f, np.array([30000, -5]), np.array([20000, 7])).kind == "unknown"
    assert _preflight.check("mul", f, np.array([M]), np.array([M])).kind == "safe"
    v = _preflight.check("div", f, np.array([1, 2, 3]), np.array([0, 5, 0]))
    assert v.events["div0"] == 2
    assert _preflight.check("div", f, np.array([9, 8]), np.array([3, 8])).kind == "certain"
    assert _preflight.check("div", f, np.array([1, 2]), np.array([3, 8])).kind == "safe"
    assert _preflight.check("sqrt", f, np.array([-1, 4, -3])).events["invalid"] == 2
    small = np.full((4, 4), 327)
    assert _preflight.check("matmul", f, small, small).kind == "safe"
    big = np.full((4, 4), 29490)
    assert _preflight.check("matmul", f, big, big).kind == "unknown"
    assert _preflight.check("fma", f, np.array([10]), np.array([10]), np.array([M])).kind == "safe"
    assert _preflight.check("add", f, np.zeros((0,), np.int64), np.zeros((0,), np.int64)).kind == "safe"


def test_chain_bound_and_wide_safety_match_the_oracle():
    from oracle import sfref
    rng = np.random.default_rng(3)
    for bits in (16, 8):
        M = (1 << (bits - 1)) - 1
        a = rng.integers(-M, M + 1, (5, 30))
        b = rng.integers(-M, M + 1, (30, 4))
        assert _preflight.chain_bound(FORMATS[bits], a, b) == sfref.chain_bound(bits, a, b)
        for mx in ("v4.9.2", "v4.8.1"):
            for scale in (1, 50):
                assert _preflight.wide_acc_safe(FORMATS[bits], a // scale, b, mx) == \
                    sfref.wide_acc_safe(bits, a // scale, b, mx)


def test_errstate_scoping_threads_and_tasks():
    assert sf.geterr() == {"over": "raise", "under": "warn", "divide": "raise", "invalid": "raise"}
    with sf.errstate(all="ignore"):
        assert set(sf.geterr().values()) == {"ignore"}
        with sf.errstate(over="warn"):
            assert sf.geterr()["over"] == "warn"
        assert sf.geterr()["over"] == "ignore"
    assert sf.geterr()["over"] == "raise"

    @sf.errstate(under="raise")
    def f():
        return sf.geterr()["under"]
    assert f() == "raise" and sf.geterr()["under"] == "warn"

    async def g():
        with sf.errstate(divide="ignore"):
            await asyncio.sleep(0)
            return sf.geterr()["divide"]
    assert asyncio.run(g()) == "ignore" and sf.geterr()["divide"] == "raise"
    with pytest.raises(ValueError):
        sf.errstate(bogus="raise")
    with pytest.raises(TypeError):
        @sf.errstate(all="ignore")
        def gen():
            yield 1


def test_config_and_accumulate_scoping():
    assert sf.getconfig()["preflight"] == "raise" and sf.getconfig()["default_device"] == "b200"
    with sf.config(preflight="warn", probe_size=8):
        assert sf.getconfig()["preflight"] == "warn" and sf.getconfig()["probe_size"] == 8
    assert sf.getconfig()["preflight"] == "raise"
    with pytest.raises(ValueError):
        sf.config(preflight="maybe")
    assert sf.getaccumulate() == "chain"
    with sf.accumulate("wide"):
        assert sf.getaccumulate() == "wide"
    assert sf.getaccumulate() == "chain"
    with pytest.raises(ValueError):
        sf.accumulate("fast")


def test_shift_validation_and_shape_errors_before_any_launch():
    a = sf.from_codes(np.ones((3, 4), np.int64), sf.sf16)
    b = sf.from_codes(np.ones((5, 2), np.int64), sf.sf16)
    with pytest.raises(sf.SFShapeError, match="not aligned"):
        a @ b
    with pytest.raises(ValueError, match="shift= only applies"):
        sf.matmul(a, a.T, shift=1)
    with pytest.raises(ValueError, match="between -32 and 31"):
        sf.matmul(a, a.T, accumulate="wide", shift=40)
    with pytest.raises(TypeError):
        sf.matmul(a, a.T, accumulate="wide", shift=True)
    with pytest.raises(sf.SFShapeError):
        sf.from_codes(np.ones(3, np.int64), sf.sf16) + sf.from_codes(np.ones(4, np.int64), sf.sf16)
    with pytest.raises(sf.SFTypeError):
        sf.asarray([0.5], dtype=sf.sf8) + "x"


def test_status_type():
    s = sf.SFStatus(saturated=3, exact=True, outputs_at_max=3)
    assert repr(s) == "SFStatus(saturated=3, underflow=0, div0=0, invalid=0, exact=True)"
    assert s.ok is False and s.known
    assert sf.SFStatus().ok is True
    assert sf.SFStatus(saturated=None).ok is None
    with warnings.catch_warnings():
        warnings.simplefilter("error")
        repr(sf.SFStatus(underflow=None))


def test_device_registry_and_attributes():
    d = sf.get_device("b200")
    assert d.sticky_flags and d.mx == "v4.9.2" and d.name == "b200"
    assert d.widths_for("matmul_wide") == tuple(range(4, 17))
    assert "b200" in sf.devices() and "host" in sf.devices()
    with pytest.raises(sf.SFUnsupportedError):
        sf.get_device("nowhere")
    mine = sf.B200Device(0, mx="v4.8.1", name="b200-v481")
    sf.register_device(mine)
    assert sf.get_device("b200-v481") is mine and mine.mx == "v4.8.1"
    with pytest.raises(ValueError):
        sf.B200Device(0, mx="v9")


@pytest.mark.parametrize("n", [0, 1, 7, 8, 1000, (1 << 20) + 3, 3 << 20, (1 << 26) + 12345])
def test_host_pipeline_cuts(n):
    """The host pipeline's chunk ranges: contiguous cover of [0, n), no chunk
    above the slot size, 16-byte aligned starts, and a short last chunk."""
    from superfloat.python_b200._hostpath import cuts
    chunk = 1 << 20
    c = cuts(n, chunk)
    assert [lo for lo, _ in c] == ([0] if c else []) + [hi for _, hi in c[:-1]]
    assert (c[-1][1] if c else 0) == n
    assert all(0 < hi - lo <= chunk and lo % 8 == 0 for lo, hi in c)
    if n > 2 * chunk:
        assert c[-1][1] - c[-1][0] <= chunk // 8
