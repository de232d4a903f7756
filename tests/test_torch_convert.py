"""sft.convert plumbing without a GPU: what gets converted, reports, configs."""
import pytest
import torch
import torch.nn as nn

import superfloat.python_b200 as sf
import superfloat.python_b200.torch as sft


class Conv1D(nn.Module):
    """The shape of Hugging Face's Conv1D (weight stored (in, out))."""

    def __init__(self, nf, nx):
        super().__init__()
        self.nf, self.nx = nf, nx
        self.weight = nn.Parameter(torch.randn(nx, nf) * 0.02)
        self.bias = nn.Parameter(torch.zeros(nf))

    def forward(self, x):
        return torch.addmm(self.bias, x.reshape(-1, self.nx), self.weight).reshape(*x.shape[:-1], self.nf)


class Net(nn.Module):
    def __init__(self):
        super().__init__()
        self.emb = nn.Embedding(50, 8)
        self.fc = nn.Linear(8, 8)
        self.c1d = Conv1D(8, 8)
        self.conv = nn.Conv2d(1, 2, 3, padding=1)
        self.grouped = nn.Conv2d(2, 2, 3, groups=2)
        self.rnn = nn.GRU(4, 4)
        self.head = nn.Linear(8, 50, bias=False)
        self.head.weight = self.emb.weight
        self.alias = self.fc


def test_convert_swaps_and_reports():
    torch.manual_seed(0)
    m = Net()
    c = sft.convert(m)
    assert isinstance(c.fc, sft.SFLinear) and isinstance(c.c1d, sft.SFHFConv1D)
    assert isinstance(c.conv, sft.SFConv2d) and isinstance(c.grouped, nn.Conv2d)
    assert c.alias is c.fc                                  # shared module converted once
    assert c.head.weight is c.emb.weight                    # tied weight kept
    assert isinstance(m.fc, nn.Linear) and not isinstance(m.fc, sft.SFLinear)   # not inplace
    rep = sft.conversion_report(c)
    kinds = dict(rep.converted)
    assert kinds["fc"] == "Linear" and kinds["c1d"] == "Conv1D (Hugging Face)" and kinds["conv"] == "Conv2d"
    assert ("alias", "fc") in rep.shared
    skipped = {n: why for n, _, why in rep.skipped}
    assert "groups=2" in skipped["grouped"] and "runs in float" in skipped["rnn"]
    assert "ConversionReport: 4 converted" in repr(rep)
    assert c.fc.sf_name == "fc" and "dtype=sf16, scale=per_tensor, headroom=bound" in repr(c.fc)


def test_keep_sf16_and_widths():
    torch.manual_seed(0)
    c = sft.convert(Net(), dtype=sf.sf8)
    rep = sft.conversion_report(c)
    assert rep.widths["head"] == 16 and rep.widths["fc"] == 8
    assert rep.kept_sf16 == [("head", "LM head (weight tied to the embeddings)")]
    c = sft.convert(Net(), dtype="sf8", keep_sf16=False, widths={"fc": "sf12"})
    assert c.fc.sf.bits == 12 and c.head.sf.bits == 8
    with pytest.raises(ValueError, match="no module named"):
        sft.convert(Net(), dtype="sf8", keep_sf16=["nope"])
    with pytest.raises(ValueError, match="no module named"):
        sft.convert(Net(), widths={"nope": 8})


def test_config_validation():
    with pytest.raises(ValueError):
        sft.SFConfig(16, "per_row")
    with pytest.raises(ValueError):
        sft.SFConfig(16, headroom="some")
    with pytest.raises(ValueError):
        sft.SFConfig(3)
    with pytest.raises(ValueError):
        sft.SFConfig(16, shift=2)
    with pytest.raises(ValueError):
        sft.SFConfig(16, accumulate="wide", shift=40)
    c = sft.convert(Net(), accumulate="wide", shift=-3, attention=False)
    with pytest.raises(sf.SFUnsupportedError, match="attention=False"):
        sft.convert(Net(), accumulate="wide")
    assert c.fc.sf.accumulate == "wide" and c.fc.sf.shift == -3


def test_lm_head_rules():
    torch.manual_seed(0)
    m = Net()
    assert sft.find_lm_heads(m) == {id(m.head): "LM head (weight tied to the embeddings)"}
    assert sft.find_lm_heads(nn.Sequential(nn.Linear(3, 3))) == {}
    assert sft.is_hf_conv1d(Conv1D(4, 3)) and not sft.is_hf_conv1d(nn.Linear(3, 4))


def test_backend_is_registered():
    import torch._dynamo
    assert "superfloat" in torch._dynamo.list_backends()
    with pytest.raises(ValueError, match="no graph"):
        if not sft.compile_reports():
            sft.compile_report()
        else:
            raise ValueError("no graph (already compiled in this process)")
