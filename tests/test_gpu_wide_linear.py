"""The wide sft path on the B200 (sf::linear_wide / sf::matmul_wide) vs the
reference, bit for bit: the reference's golden cases and its seeded runs
(tests/golden/make_golden_wide.py: guard raises, redos, clamped bias codes,
flushes, explicit shifts, both chips, widths 4..16), GPT-2-small converted
with accumulate="wide" (every layer's output hash and status, the logits),
and larger random layers and batched activation matmuls against the oracle."""
import hashlib
import json
import os
import warnings

import numpy as np
import pytest
import torch

from conftest import GOLDEN
from oracle import native, sfref
import superfloat.python_b200.torch as sft
from superfloat.python_b200.torch import _wide

pytestmark = pytest.mark.gpu
META = json.load(open(os.path.join(GOLDEN, "wide_layers.json")))
ARR = np.load(os.path.join(GOLDEN, "wide_layers.npz"))
CASES = META["spec"] + META["runs"]
KEYS = ("saturated", "exact", "underflow", "input_underflow", "weight_underflow", "bias_saturated", "headroom_bits",
        "outputs", "act_scale", "accumulate", "shift_min", "shift_max", "h", "redone", "flushed", "acc_clipped",
        "guard_raised")


def sha(t):
    return hashlib.sha256(t.detach().cpu().contiguous().numpy().tobytes()).hexdigest()


def check_status(got, want, what):
    for k in KEYS:
        if k in want:
            assert getattr(got, k) == want[k], (what, k, getattr(got, k), want[k])


@pytest.mark.parametrize("case", CASES, ids=[c["key"] for c in CASES])
def test_reference_cases(gpu, case):
    k = case["key"]
    x = torch.from_numpy(ARR[k + "__x"])
    w = torch.from_numpy(ARR[k + "__w"])
    b = torch.from_numpy(ARR[k + "__b"]) if case["has_bias"] else None
    r = _wide.wide_linear(x, w, b, case["bits"], case.get("shift"), out_dtype=torch.float64,
                          mx=case.get("mx") or _wide.MX_DEFAULT)
    np.testing.assert_array_equal(r.y.cpu().numpy(), ARR[k + "__y"])
    check_status(r, case["status"], k)


@pytest.mark.parametrize("bits", [16, 12, 8, 4])
def test_random_layers_against_the_oracle(gpu, bits, rng):
    for (R, K, N), bias in (((300, 1000, 200), True), ((129, 64, 257), False), ((4, 4096, 9), True)):
        x = rng.standard_normal((R, K)) * np.exp(rng.uniform(-3, 3, (R, 1)))
        w = rng.standard_normal((N, K)) * 0.05
        b = rng.standard_normal(N) * 0.1 if bias else None
        y, st = sfref.wide_linear(x, w, b, bits, acc_fn=native.wide_acc)
        r = _wide.wide_linear(torch.from_numpy(x), torch.from_numpy(w), None if b is None else torch.from_numpy(b),
                              bits, out_dtype=torch.float64)
        np.testing.assert_array_equal(r.y.cpu().numpy(), y, err_msg=f"sf{bits} {R}x{K}x{N}")
        check_status(r, st, f"sf{bits} {R}x{K}x{N}")


def test_float32_output_rounds_once(gpu, rng):
    x = rng.standard_normal((40, 300)).astype(np.float32)
    w = rng.standard_normal((30, 300)) * 0.05
    y, _ = sfref.wide_linear(x.astype(np.float64), w, None, 16, acc_fn=native.wide_acc)
    r = _wide.wide_linear(torch.from_numpy(x), torch.from_numpy(w), None, 16)
    assert r.y.dtype == torch.float32
    np.testing.assert_array_equal(r.y.cpu().numpy(), y.astype(np.float32))


def test_activation_matmul_batched(gpu, rng):
    a = rng.standard_normal((3, 17, 70))
    b = rng.standard_normal((3, 70, 23)) * np.exp(rng.uniform(-2, 2, (3, 1, 23)))
    r = _wide.wide_matmul(torch.from_numpy(a), torch.from_numpy(b), 16, out_dtype=torch.float64)
    tot = dict.fromkeys(("saturated", "underflow", "redone", "flushed", "input_underflow", "outputs"), 0)
    for i in range(3):
        y, st = sfref.wide_matmul(a[i], b[i], 16, acc_fn=native.wide_acc)
        np.testing.assert_array_equal(r.y[i].cpu().numpy(), y)
        for k in tot:
            tot[k] += st[k]
    for k, v in tot.items():
        assert getattr(r, k) == v, k
    y, st = sfref.wide_matmul(a[0], b[0], 8, shift=-4, acc_fn=native.wide_acc)
    r = _wide.wide_matmul(torch.from_numpy(a[0]), torch.from_numpy(b[0]), 8, shift=-4, out_dtype=torch.float64)
    np.testing.assert_array_equal(r.y.cpu().numpy(), y)
    check_status(r, st, "shift -4")


def test_empty_and_zero_shapes(gpu):
    r = _wide.wide_linear(torch.zeros(0, 5), torch.ones(3, 5), None, 16)
    assert r.y.shape == (0, 3) and r.outputs == 0 and r.shift_min is None
    r = _wide.wide_linear(torch.zeros(4, 5), torch.zeros(3, 5), torch.zeros(3), 16, out_dtype=torch.float64)
    assert not r.y.any() and r.saturated == 0 and r.redone == 0


def _gpt2():
    from transformers import GPT2Config, GPT2LMHeadModel
    torch.manual_seed(0)
    cfg = GPT2Config(n_layer=12, n_embd=768, n_head=12, n_inner=3072, vocab_size=50257, n_positions=1024)
    return GPT2LMHeadModel(cfg).eval()


def test_gpt2_wide_matches_the_reference(gpu):
    """GPT-2-small with accumulate="wide", float parts on the CPU as the
    reference ran them: every layer's input and output hash and status, the
    recorded first-block layers fed the reference's inputs, and the logits."""
    g = META["gpt2"]
    model = sft.convert(_gpt2(), dtype="sf16", accumulate="wide", attention=False)
    ids = torch.from_numpy(ARR[g["ids"]])
    seen = []
    hooks = [m.register_forward_hook(lambda mod, i, o: seen.append((mod.sf_name, sha(i[0]), sha(o))))
             for m in model.modules() if hasattr(m, "sf_name")]
    with torch.no_grad():
        sft.reset_status()
        y = model(ids)
    for h in hooks:
        h.remove()
    st = sft.last_status(model)
    assert len(seen) == len(g["layers"]) == 49
    for (name, in_sha, out_sha), lay in zip(seen, g["layers"]):
        assert name == lay["name"]
        assert in_sha == lay["in_sha"], f"{name}: the host float path gave a different input"
        assert out_sha == lay["out_sha"], name
        check_status(st[name], lay["status"], name)
    assert sha(y.logits) == g["logits_sha"]
    mods = {m.sf_name: m for m in model.modules() if hasattr(m, "sf_name")}
    with torch.no_grad():
        for lay in (x for x in g["layers"] if x.get("recorded")):
            out = mods[lay["name"]](torch.from_numpy(ARR[lay["key"] + "__in"]))
            np.testing.assert_array_equal(out.numpy(), ARR[lay["key"] + "__out"])


def test_gpt2_wide_compiled_on_the_gpu(gpu):
    torch._dynamo.reset()
    model = sft.convert(_gpt2(), dtype="sf16", accumulate="wide", attention=False).cuda()
    ids = torch.randint(0, 50257, (2, 32), generator=torch.Generator().manual_seed(1)).cuda()
    with torch.no_grad():
        eager = model(ids).logits
        with warnings.catch_warnings():
            warnings.simplefilter("ignore")
            out = torch.compile(model, backend="superfloat")(ids).logits
    assert torch.equal(out, eager)
    st = sft.last_status(model)
    assert len(st) == 49 and all(s.accumulate == "wide" and s.placement == "b200" for s in st.values())
    torch._dynamo.reset()
