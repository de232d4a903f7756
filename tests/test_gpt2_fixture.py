"""The GPT-2 fixtures' inputs come back from their seeds on this machine (no
GPU): the float modules recompute block 0's c_attn input of the 8 x 512
batch and of the 64-token sequence with the hashes the reference recorded,
so the GPU tests feed the reference's exact inputs."""
import hashlib

import torch

from conftest import golden

G = golden("gpt2_64.json")


def sha(t):
    return hashlib.sha256(t.detach().contiguous().numpy().tobytes()).hexdigest()


def test_block0_inputs_reproduce():
    from transformers import GPT2Config, GPT2LMHeadModel
    torch.manual_seed(0)
    model = GPT2LMHeadModel(GPT2Config(**G["config"])).eval()
    tr = model.transformer
    for ids_shape, want in ((G["c_attn_8x512"]["ids_shape"], G["c_attn_8x512"]["in_sha"]),
                            (G["seq64"]["ids_shape"], G["seq64"]["layers"][0]["in_sha"])):
        ids = torch.randint(0, 50257, tuple(ids_shape), generator=torch.Generator().manual_seed(0))
        with torch.no_grad():
            pos = torch.arange(ids.shape[1]).unsqueeze(0)
            x = tr.h[0].ln_1(tr.drop(tr.wte(ids) + tr.wpe(pos)))
        assert sha(x) == want, ids_shape


def test_fixture_covers_every_layer():
    layers = G["seq64"]["layers"]
    assert len(layers) == 49 and layers[-1]["name"] == "lm_head"
    assert {lay["kind"] for lay in layers} == {"SFHFConv1D", "SFLinear"}
    assert G["c_attn_8x512"]["status"]["outputs"] == 4096 * 2304
