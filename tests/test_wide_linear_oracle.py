"""The oracle's wide sft linear (exponents, guard, shift rule, bias after
POP, redo) against the reference: its own golden cases
(spec/golden/wide/sft_wide.json) and its recorded runs on seeded inputs
(tests/golden/wide_layers.*), every float64 output and every status field."""
import json
import os

import numpy as np
import pytest

from oracle import native, sfref

HERE = os.path.join(os.path.dirname(__file__), "golden")
META = json.load(open(os.path.join(HERE, "wide_layers.json")))
ARR = np.load(os.path.join(HERE, "wide_layers.npz"))
CASES = [("spec", c) for c in META["spec"]] + [("runs", c) for c in META["runs"]]


@pytest.mark.parametrize("grp,case", CASES, ids=[c["key"] for _, c in CASES])
def test_wide_linear_matches_reference(grp, case):
    k = case["key"]
    b = ARR[k + "__b"] if case["has_bias"] else None
    y, st = sfref.wide_linear(ARR[k + "__x"], ARR[k + "__w"], b, case["bits"], case.get("shift"),
                              case.get("mx") or sfref.MX_DEFAULT, acc_fn=native.wide_acc)
    np.testing.assert_array_equal(y, ARR[k + "__y"])
    for key, want in case["status"].items():
        if key in st:
            assert st[key] == want, (k, key, st[key], want)


def test_h_table_and_pow2_exp():
    assert [sfref.h_for(k) for k in (0, 1, 15, 16, 63, 64, 768, 3072, 4096)] == [0, 0, 0, 0, 0, 1, 2, 3, 4]
    assert sfref.pow2_exp(np.array([0.0, 0.5, 0.75, 1.0, 3.0, 2.0 ** -30])).tolist() == [0, 0, 0, 1, 2, -29]
