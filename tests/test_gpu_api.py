"""The array API on the B200 target: results equal the oracle, status is
exact (sticky per-output events), the error policy and the pre-flight gate
behave as the reference's flagged target does (tests/test_1_1_3_matmul_device.py
of the reference)."""
import warnings

import numpy as np
import pytest

import superfloat.python_b200 as sf
from oracle import native, sfref

pytestmark = pytest.mark.gpu
DEV = "b200"


def launches():
    return sf.get_device(DEV).launches


def test_heavy_ops_equal_the_oracle(gpu):
    rng = np.random.default_rng(3)
    for shape in [(64,), (8, 9), (3, 4, 5)]:
        ka = rng.integers(-32767, 32768, shape)
        kb = rng.integers(-32767, 32768, shape)
        kb.reshape(-1)[0] = 0
        a, b = sf.from_codes(ka, sf.sf16, device=DEV), sf.from_codes(kb, sf.sf16, device=DEV)
        with sf.errstate(all="ignore"), sf.config(preflight="ignore", suspect="ignore"):
            cases = [(a + b, sfref.add(16, ka, kb)), (a - b, sfref.sub(16, ka, kb)),
                     (a * b, sfref.mul(16, ka, kb)), (a / b, sfref.div(16, ka, kb)),
                     (sf.fma(a, b, b), sfref.fma(16, ka, kb, kb)), (-a, sfref.neg(16, ka)),
                     (abs(a), sfref.abs_(16, ka)), (a ** 3, sfref.pow_int(16, ka, 3)),
                     (sf.sqrt(a), sfref.sqrt(16, ka))]
        for got, (want, ev) in cases:
            assert got.device == DEV and got.codes.tolist() == want.tolist()
            assert got.status.exact
            assert got.status.saturated == int(np.count_nonzero(ev.get("overflow", False)))
            assert got.status.underflow == int(np.count_nonzero(ev.get("underflow", False)))


def test_host_arrays_run_on_the_target_with_light_semantics(gpu):
    a = sf.asarray([0.25, 0.125], dtype=sf.sf16)
    n0 = launches()
    y = a + a
    assert y.device == "host" and y.status is None and y.codes.tolist() == [16384, 8192]
    with pytest.raises(sf.SFOverflowError, match="overflow in 1 of 2"):
        sf.asarray([0.75, 0.25], dtype=sf.sf16) + sf.asarray([0.75, 0.25], dtype=sf.sf16)
    with pytest.warns(sf.SFUnderflowWarning, match="underflow in 1 of 1"):
        sf.from_codes(np.array([3]), sf.sf16) * sf.from_codes(np.array([5]), sf.sf16)
    assert launches() >= n0 + 2


def test_flagged_status_and_policy(gpu):
    a = sf.array([0.75, 0.25], dtype=sf.sf16, device=DEV)
    with pytest.raises(sf.SFOverflowError, match="status.saturated"):
        a + a
    with sf.errstate(over="ignore"):
        y = a + a
    assert y.status.exact and y.status.saturated == 1 and y.status.ok is False
    assert y.status == sf.SFStatus(saturated=1, div0=0, invalid=0, exact=True, outputs_at_max=1, underflow=0)
    # an exact +-max input from a non-saturating add is not a saturation
    s = sf.array([0.25, -0.5], dtype=sf.sf16, device=DEV) + sf.from_codes(np.array([32767 - 8192, 100]),
                                                                           sf.sf16, device=DEV)
    assert s.codes.tolist() == [32767, -16384 + 100] and s.status.saturated == 0 and s.status.outputs_at_max == 1
    # div0 / invalid: read off the inputs before the launch
    b = sf.array([0.5, 0, 0.25, 0], dtype=sf.sf16, device=DEV)
    a4 = sf.array([0.75, 0.25, -0.1, 0.5], dtype=sf.sf16, device=DEV)
    n0 = launches()
    with pytest.raises(sf.SFZeroDivisionError, match="status.div0"):
        a4 / b
    assert launches() == n0
    with sf.errstate(divide="ignore", over="ignore"):
        q = a4 / b
    assert q.status.div0 == 2 and q.codes.tolist()[1] == 32767 and q.codes.tolist()[3] == 32767
    assert q.status.saturated == 1                        # 0.75 / 0.5
    n = sf.array([0.25, -0.25], dtype=sf.sf16, device=DEV)
    with pytest.raises(sf.SFInvalidError, match="status.invalid"):
        sf.sqrt(n)
    with sf.errstate(invalid="ignore"):
        r = sf.sqrt(n)
    assert r.status == sf.SFStatus(saturated=0, div0=0, invalid=1, exact=True)
    assert r.codes.tolist() == [16384, 0]


def test_preflight_refuses_certain_saturation_without_launch(gpu):
    big = sf.full((4, 4), 0.9, sf.sf16, device=DEV)
    n0 = launches()
    with pytest.raises(sf.SFOverflowError, match="pre-flight"):
        big + big
    with pytest.raises(sf.SFOverflowError, match="pre-flight"):
        big / sf.full((4, 4), 0.5, sf.sf16, device=DEV)
    assert launches() == n0
    with sf.errstate(over="ignore"):
        with warnings.catch_warnings(record=True) as w:
            warnings.simplefilter("always")
            big @ big
    assert launches() == n0 + 1 and any(issubclass(x.category, sf.SFPreflightWarning) for x in w)
    with sf.config(suspect="raise"):
        with pytest.raises(sf.SFOverflowError, match="suspected"):
            big @ big
    with sf.config(suspect="verify"):
        with pytest.raises(sf.SFOverflowError, match="host replay"):
            big @ big
    assert launches() == n0 + 1
    with sf.config(preflight="ignore"), sf.errstate(over="ignore"):
        y = big + big
    assert y.status.saturated == 16 and y.status.outputs_at_max == 16 and launches() == n0 + 2


def test_matmul_api_chain_and_wide(gpu, rng):
    A = rng.integers(-3000, 3001, (6, 40))
    B = rng.integers(-32767, 32768, (40, 5))
    a, b = sf.from_codes(A, sf.sf16, device=DEV), sf.from_codes(B, sf.sf16, device=DEV)
    with sf.errstate(all="ignore"), sf.config(suspect="ignore"):
        y = a @ b
        want, ev = sfref.matmul_chain(16, A, B)
        assert y.codes.tolist() == want.tolist() and y.status.exact
        assert y.status.saturated == int(ev["overflow"].sum()) and y.status.underflow == int(ev["underflow"].sum())
        w = sf.matmul(a, b, accumulate="wide", shift=-2)
        want, ev = sfref.matmul_wide(16, A, B, -2)
        assert w.codes.tolist() == want.tolist() and w.status.saturated == int(ev["overflow"].sum())
        sh = rng.integers(-5, 3, (6, 1))
        w = sf.matmul(a, b, accumulate="wide", shift=sh)
        want, _ = sfref.matmul_wide(16, A, B, sh)
        assert w.codes.tolist() == want.tolist()
        with sf.accumulate("wide"):
            w2 = a @ b
        want, _ = sfref.matmul_wide(16, A, B, 0)
        assert w2.codes.tolist() == want.tolist()
        v = sf.dot(a[0], b[:, 0])
        assert v.codes.tolist() == sfref.matmul_chain(16, A[:1], B[:, :1])[0][0, 0].tolist()
        d = sf.from_codes(rng.integers(-32767, 32768, (5,)), sf.sf16, device=DEV)
        z = sf.addmm(a, b, d)
        want, _ = sfref.add(16, sfref.matmul_chain(16, A, B)[0], d.codes[None, :])
        assert z.codes.tolist() == want.tolist()


def test_mixed_widths_widen(gpu):
    a8 = sf.from_codes(np.array([5, -7, 100]), sf.sf8, device=DEV)
    b16 = sf.from_codes(np.array([1000, 2000, -3000]), sf.sf16, device=DEV)
    y = a8 + b16
    assert y.dtype is sf.sf16
    want, _ = sfref.add(16, np.array([5, -7, 100]) << 8, np.array([1000, 2000, -3000]))
    assert y.codes.tolist() == want.tolist()


def test_v481_device_wide(gpu, rng):
    dev = sf.B200Device(0, mx="v4.8.1", name="b200-v481-api")
    sf.register_device(dev)
    A = rng.integers(-32767, 32768, (4, 100))
    B = rng.integers(-32767, 32768, (100, 3))
    with sf.errstate(all="ignore"):
        y = sf.matmul(sf.from_codes(A, sf.sf16, device=dev.name), sf.from_codes(B, sf.sf16, device=dev.name),
                      accumulate="wide", shift=-3)
    want, ev = sfref.matmul_wide(16, A, B, -3, "v4.8.1", acc_fn=native.wide_acc)
    assert y.codes.tolist() == want.tolist() and y.status.saturated == int(ev["overflow"].sum())
