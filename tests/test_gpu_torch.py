"""Converted layers on the B200 vs the reference's sf.torch, bit for bit.

The fixtures (tests/golden/make_golden_torch.py) hold, for seeded models the
reference converted and ran on the CPU, each SF layer's input, output and
status.  Each layer here gets the same input and must give the same float32
output and the same status fields, including the activation scale.  The
whole models also run end to end with the float parts on the CPU (as the
reference runs them) and through torch.compile(backend="superfloat").
"""
import hashlib
import os
import warnings

import numpy as np
import pytest
import torch
import torch.nn as nn
import torch.nn.functional as F

from conftest import GOLDEN, golden
import superfloat.python_b200 as sf
import superfloat.python_b200.torch as sft

pytestmark = pytest.mark.gpu
META = golden("torch_layers.json")
ARR = np.load(os.path.join(GOLDEN, "torch_layers.npz"))
STATUS_KEYS = ("op", "dtype", "outputs", "saturated", "exact", "underflow", "input_underflow", "weight_underflow",
               "bias_saturated", "headroom_bits", "act_scale")


def sha(t):
    return hashlib.sha256(t.detach().cpu().contiguous().numpy().tobytes()).hexdigest()


class Attention(nn.Module):
    def __init__(self, d=16):
        super().__init__()
        self.q, self.k, self.v, self.o = (nn.Linear(d, d) for _ in range(4))
        self.d = d

    def forward(self, x):
        q, k, v = self.q(x), self.k(x), self.v(x)
        scores = sft.matmul(q, k.transpose(-1, -2), name="attn.qk") / self.d ** 0.5
        return self.o(sft.matmul(torch.softmax(scores, dim=-1), v, name="attn.wv"))


class CNN(nn.Module):
    def __init__(self):
        super().__init__()
        self.c1 = nn.Conv2d(1, 4, 3, padding=1)
        self.fc = nn.Linear(4 * 4 * 4, 3)

    def forward(self, x):
        x = F.max_pool2d(torch.relu(self.c1(x)), 2)
        return self.fc(x.flatten(1))


MAKE = {"mlp": lambda: nn.Sequential(nn.Linear(12, 24), nn.ReLU(), nn.Linear(24, 6)), "cnn": CNN,
        "attention": Attention}


def _check_status(got, want, what):
    for k in STATUS_KEYS:
        assert getattr(got, k) == want[k], (what, k, getattr(got, k), want[k])


def _layers_by_name(model):
    return {m.sf_name: m for m in model.modules() if hasattr(m, "sf_name")}


@pytest.mark.parametrize("case", [c["tag"] for c in META["cases"]])
def test_small_models_layer_by_layer(gpu, case):
    c = next(x for x in META["cases"] if x["tag"] == case)
    torch.manual_seed(0)
    model = sft.convert(MAKE[c["arch"]](), headroom=c["headroom"], scale=c["scale"])
    x = torch.from_numpy(ARR[c["x"]])
    assert torch.equal(x, torch.randn(*x.shape) * 3)          # the same seeded input
    mods = _layers_by_name(model)
    with torch.no_grad():
        for lay in c["layers"]:
            xin = torch.from_numpy(ARR[lay["key"] + "__in"])
            want = ARR[lay["key"] + "__out"]
            with sft.capture_status() as st:
                if lay["name"] in mods:
                    y = mods[lay["name"]](xin)
                else:                                            # the attention block's two sft.matmul calls
                    continue
            assert np.array_equal(y.numpy(), want), (case, lay["name"])
            _check_status(st[lay["name"]], lay["status"], (case, lay["name"]))
        sft.reset_status()
        y = model(x)
    assert sha(y) == c["y_sha"], case
    st = sft.last_status()
    for lay in c["layers"]:
        _check_status(st[lay["name"]], lay["status"], (case, lay["name"], "whole model"))


def test_compiled_equals_eager_and_reports(gpu):
    torch._dynamo.reset()
    torch.manual_seed(0)
    model = sft.convert(Attention())
    x = torch.randn(2, 7, 16) * 3
    with torch.no_grad():
        eager = model(x)
        st_e = sft.last_status(model)
        n0 = sf.get_device("b200").launches
        compiled = torch.compile(model, backend="superfloat")
        out = compiled(x)
        st_c = sft.last_status(model)
    assert torch.equal(out, eager)
    rep = sft.compile_report()
    assert sorted(n for _, _, n, _ in rep.on_device) == ["attn.qk", "attn.wv", "k", "o", "q", "v"]
    assert rep.coverage == 1.0 and "6 SF op(s) on device" in repr(rep)
    for name, s in st_c.items():
        assert s.placement == "b200" and s.saturated == 0 and s.exact and s.act_scale == st_e[name].act_scale
    torch._dynamo.reset()
    p = sft.convert(nn.Sequential(nn.Linear(4, 4)))
    cp = torch.compile(p, backend="superfloat")
    with pytest.raises(Exception, match="inference-only"):
        cp(torch.randn(3, 4))
    torch._dynamo.reset()


def test_training_gradient_is_straight_through(gpu):
    torch.manual_seed(0)
    lin = nn.Linear(6, 3)
    m = sft.convert(nn.Sequential(lin))
    x = torch.randn(5, 6, requires_grad=True)
    m(x).sum().backward()
    assert x.grad is not None and m[0].weight.grad is not None and m[0].bias.grad is not None
    assert torch.allclose(m[0].bias.grad, torch.full((3,), 5.0))


def _gpt2():
    from transformers import GPT2Config, GPT2LMHeadModel
    torch.manual_seed(0)
    cfg = GPT2Config(**META["gpt2"]["config"])
    return GPT2LMHeadModel(cfg).eval()


def test_gpt2_layers_match_the_reference(gpu):
    g = META["gpt2"]
    model = sft.convert(_gpt2(), dtype="sf16")
    mods = _layers_by_name(model)
    assert len(mods) == 49 and len(g["layers"]) == 49
    rec = [lay for lay in g["layers"] if lay["recorded"]]
    assert len(rec) == 5
    with torch.no_grad():
        for lay in rec:
            xin = torch.from_numpy(ARR[lay["key"] + "__in"])
            with sft.capture_status() as st:
                y = mods[lay["name"]](xin)
            assert sha(y) == lay["out_sha"], lay["name"]
            _check_status(st[lay["name"]], lay["status"], lay["name"])


def test_gpt2_end_to_end_on_the_host_float_path(gpu):
    """The whole model with its float parts on the CPU, as the reference ran
    it: every layer's input, output and status, and the logits."""
    g = META["gpt2"]
    model = sft.convert(_gpt2(), dtype="sf16")
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
    for (name, in_sha, out_sha), lay in zip(seen, g["layers"]):
        assert name == lay["name"]
        assert in_sha == lay["in_sha"], f"{name}: the host float path gave a different input"
        assert out_sha == lay["out_sha"], name
        _check_status(st[name], lay["status"], name)
    assert sha(y.logits) == g["logits_sha"]


def test_gpt2_on_the_gpu_compiled(gpu):
    """GPT-2-small converted, on the GPU, through torch.compile: every layer
    on the device, headroom proves no saturation, compiled == eager."""
    torch._dynamo.reset()
    model = sft.convert(_gpt2(), dtype="sf16").cuda()
    ids = torch.randint(0, 50257, (2, 64), generator=torch.Generator().manual_seed(1)).cuda()
    with torch.no_grad():
        eager = model(ids).logits
        compiled = torch.compile(model, backend="superfloat")
        with warnings.catch_warnings():
            warnings.simplefilter("ignore")
            out = compiled(ids).logits
    assert torch.equal(out, eager)
    st = sft.last_status(model)
    assert len(st) == 49 and all(s.saturated == 0 and s.exact and s.placement == "b200" for s in st.values())
    torch._dynamo.reset()


@pytest.mark.parametrize("case", [c["tag"] for c in META["cases"] if c["headroom"] == "bound"])
def test_prepared_layers_search_the_scale_on_the_device(gpu, case):
    """A layer's second call (weight and bias prepared) runs the scale search,
    bias codes and chain on the device with one host read: the same output
    and status as the reference."""
    from superfloat.python_b200.torch import _core
    c = next(x for x in META["cases"] if x["tag"] == case)
    torch.manual_seed(0)
    model = sft.convert(MAKE[c["arch"]](), headroom=c["headroom"], scale=c["scale"])
    mods = _layers_by_name(model)
    with torch.no_grad():
        for lay in c["layers"]:
            xin = torch.from_numpy(ARR[lay["key"] + "__in"])
            mods[lay["name"]](xin)                              # prepares the weight and bias
            before = _core.device_path_calls
            with sft.capture_status() as st:
                y = mods[lay["name"]](xin)
            assert _core.device_path_calls == before + 1, lay["name"]
            np.testing.assert_array_equal(y.numpy(), ARR[lay["key"] + "__out"], err_msg=lay["name"])
            _check_status(st[lay["name"]], lay["status"], lay["name"])


def test_gpt2_second_forward_on_the_device_path(gpu):
    """GPT-2-small twice: the second forward's 49 layers all take the device
    path and match the reference's layer outputs, statuses and logits."""
    from superfloat.python_b200.torch import _core
    g = META["gpt2"]
    model = sft.convert(_gpt2(), dtype="sf16")
    ids = torch.from_numpy(ARR[g["ids"]])
    with torch.no_grad():
        model(ids)
        before = _core.device_path_calls
        seen = []
        hooks = [m.register_forward_hook(lambda mod, i, o: seen.append((mod.sf_name, sha(o))))
                 for m in model.modules() if hasattr(m, "sf_name")]
        sft.reset_status()
        y = model(ids)
        for h in hooks:
            h.remove()
    assert _core.device_path_calls == before + 49
    st = sft.last_status(model)
    for (name, out_sha), lay in zip(seen, g["layers"]):
        assert out_sha == lay["out_sha"], name
        _check_status(st[name], lay["status"], name)
    assert sha(y.logits) == g["logits_sha"]


def test_nan_input_on_a_prepared_layer_takes_the_policy(gpu):
    lin = sft.convert(nn.Sequential(nn.Linear(8, 4)))[0]
    x = torch.randn(3, 8)
    with torch.no_grad():
        lin(x)
        x[1, 2] = float("nan")
        with pytest.raises(sf.SFInvalidError):
            lin(x)
        with sf.errstate(invalid="ignore"):
            y = lin(x)
    assert torch.isfinite(y).all()
