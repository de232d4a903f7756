"""GPT-2-small converted (chain, sf16, headroom "bound") against the
reference's own run beyond 8 tokens (tests/golden/gpt2_64.json, made by
tests/golden/make_golden_gpt2.py with the reference's sf.torch):

* one sequence of 64 tokens, eager and through
  torch.compile(backend="superfloat"): every SF layer's input, output and
  status, and the logits, with the float parts on the CPU as the reference
  ran them (so every layer's input is the reference's, bit for bit);
* block 0's c_attn at the full shape of the 8 x 512-token batch (4096 x 768
  activations), from CPU inputs and from CUDA inputs.
"""
import hashlib
import warnings

import pytest
import torch

from conftest import golden
import superfloat.python_b200.torch as sft

pytestmark = pytest.mark.gpu
G = golden("gpt2_64.json")
STATUS_KEYS = ("op", "dtype", "outputs", "saturated", "exact", "underflow", "input_underflow", "weight_underflow",
               "bias_saturated", "headroom_bits", "act_scale")


def sha(t):
    return hashlib.sha256(t.detach().cpu().contiguous().numpy().tobytes()).hexdigest()


def _model():
    from transformers import GPT2Config, GPT2LMHeadModel
    torch.manual_seed(0)
    return sft.convert(GPT2LMHeadModel(GPT2Config(**G["config"])).eval(), dtype="sf16")


def _check_status(got, want, what):
    for k in STATUS_KEYS:
        assert getattr(got, k) == want[k], (what, k, getattr(got, k), want[k])


def _run_and_check(model, fn):
    g = G["seq64"]
    ids = torch.randint(0, 50257, tuple(g["ids_shape"]), generator=torch.Generator().manual_seed(0))
    seen = []
    hooks = [m.register_forward_hook(lambda mod, i, o: seen.append((mod.sf_name, sha(i[0]), sha(o))))
             for m in model.modules() if hasattr(m, "sf_name")]
    with torch.no_grad(), warnings.catch_warnings():
        warnings.simplefilter("ignore")
        sft.reset_status()
        logits = fn(ids).logits
    for h in hooks:
        h.remove()
    st = sft.last_status(model)
    assert len(st) == 49 and all(s.placement == "b200" for s in st.values())
    for lay in g["layers"]:
        _check_status(st[lay["name"]], lay["status"], lay["name"])
    if seen:                                   # eager: the hooks saw every layer call in order
        assert [n for n, _, _ in seen] == [lay["name"] for lay in g["layers"]]
        for (name, in_sha, out_sha), lay in zip(seen, g["layers"]):
            assert in_sha == lay["in_sha"], f"{name}: the host float path gave a different input"
            assert out_sha == lay["out_sha"], name
    assert sha(logits) == g["logits_sha"]


def test_gpt2_64_tokens_eager(gpu):
    model = _model()
    _run_and_check(model, model)


def test_gpt2_64_tokens_compiled(gpu):
    torch._dynamo.reset()
    model = _model()
    n0 = len(sft.compile_reports())
    compiled = torch.compile(model, backend="superfloat")
    _run_and_check(model, compiled)
    reps = sft.compile_reports()[n0:]
    # dynamo compiles a block's graph once and reuses it for the 12 blocks (and some
    # graphs between breaks hold only float ops), so the reports hold fewer SF nodes
    # than layers: none of them was left on the host
    assert sum(len(r.on_device) for r in reps) > 0 and not any(r.host_emulated for r in reps)
    torch._dynamo.reset()


def _block0_input(model, ids):
    tr = model.transformer
    pos = torch.arange(ids.shape[1]).unsqueeze(0)
    return tr.h[0].ln_1(tr.drop(tr.wte(ids) + tr.wpe(pos)))


def test_c_attn_at_the_8x512_shape(gpu):
    c = G["c_attn_8x512"]
    model = _model()
    ids = torch.randint(0, 50257, tuple(c["ids_shape"]), generator=torch.Generator().manual_seed(0))
    layer = model.transformer.h[0].attn.c_attn
    assert layer.sf_name == c["name"]
    with torch.no_grad():
        x = _block0_input(model, ids)
        assert list(x.shape) == c["in_shape"] and sha(x) == c["in_sha"]
        for inp in (x, x.cuda()):                 # host tensors, then device tensors
            with sft.capture_status() as st:
                y = layer(inp)
            assert y.device == inp.device
            assert sha(y) == c["out_sha"]
            _check_status(st[layer.sf_name], c["status"], layer.sf_name)
