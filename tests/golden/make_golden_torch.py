"""Regenerate tests/golden/torch_*.{json,npz} from the reference's sf.torch (CPU).

    SF_CACHE_DIR=/tmp/sfcache python tests/golden/make_golden_torch.py [reference_root]

For each seeded model converted with the reference's ``sft.convert`` and run
eagerly on the CPU, records every SF layer's input and output (float32) and
its ``SFLayerStatus``, plus the model output.  The layer-level records let a
test feed the exact same inputs to each converted layer on the B200, so
parity does not depend on the host's float kernels between layers.

Models: an MLP, a CNN and a small attention block (headroom "bound" and
"none", per-tensor and per-channel scales), and the GPT-2-small architecture
(12 layers, d_model 768, 12 heads, FFN 3072, vocab 50257; random init,
torch.manual_seed(0)) on one sequence of 8 token ids.
"""
from __future__ import annotations

import hashlib
import json
import os
import sys

import numpy as np

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
from _refroot import reference_root  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))


def sha(t) -> str:
    return hashlib.sha256(t.detach().contiguous().numpy().tobytes()).hexdigest()


def main(ref: str | None = None) -> None:
    ref = reference_root(ref)
    sys.path.insert(0, os.path.join(ref, "src"))
    os.environ.setdefault("SF_CACHE_DIR", "/tmp/sf_cache_golden")
    import torch
    import torch.nn as nn
    import torch.nn.functional as F
    import sf.torch as sft          # the reference

    arrays = {}
    meta = {"cases": []}

    def capture(model, x, tag):
        recs = []
        hooks = []
        for name, m in model.named_modules():
            if hasattr(m, "sf_name"):
                def hook(mod, inp, out, name=name):
                    recs.append((mod.sf_name, type(mod).__name__, inp[0].detach().clone(), out.detach().clone()))
                hooks.append(m.register_forward_hook(hook))
        sft.reset_status()
        with torch.no_grad():
            y = model(x)
        for h in hooks:
            h.remove()
        st = sft.last_status(model)
        layers = []
        for i, (name, kind, xin, yout) in enumerate(recs):
            key = f"{tag}__{i}"
            arrays[key + "__in"] = xin.numpy()
            arrays[key + "__out"] = yout.numpy()
            s = st[name]
            layers.append({"name": name, "kind": kind, "key": key, "in_shape": list(xin.shape),
                           "status": {k: getattr(s, k) for k in ("op", "dtype", "outputs", "saturated", "exact",
                                                                 "underflow", "input_underflow", "weight_underflow",
                                                                 "bias_saturated", "headroom_bits", "act_scale")}})
        return y, layers

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

    models = {
        "mlp": (lambda: nn.Sequential(nn.Linear(12, 24), nn.ReLU(), nn.Linear(24, 6)), (16, 12)),
        "cnn": (CNN, (5, 1, 8, 8)),
        "attention": (Attention, (2, 7, 16)),
    }
    for arch, (make, shape) in models.items():
        for headroom in ("bound", "none"):
            for scale in ("per_tensor", "per_channel"):
                torch.manual_seed(0)
                model = sft.convert(make(), headroom=headroom, scale=scale)
                x = torch.randn(*shape) * 3
                tag = f"{arch}_{headroom}_{scale}"
                arrays[tag + "__x"] = x.numpy()
                y, layers = capture(model, x, tag)
                meta["cases"].append({"tag": tag, "arch": arch, "headroom": headroom, "scale": scale,
                                      "x": tag + "__x", "y_sha": sha(y), "layers": layers})

    from transformers import GPT2Config, GPT2LMHeadModel
    torch.manual_seed(0)
    cfg = GPT2Config(n_layer=12, n_embd=768, n_head=12, n_inner=3072, vocab_size=50257, n_positions=1024)
    gpt = GPT2LMHeadModel(cfg).eval()
    conv = sft.convert(gpt, dtype="sf16")
    ids = torch.randint(0, 50257, (1, 8), generator=torch.Generator().manual_seed(0))
    y, layers = capture(conv, ids, "gpt2")
    arrays["gpt2__ids"] = ids.numpy()
    meta["gpt2"] = {"config": {"n_layer": 12, "n_embd": 768, "n_head": 12, "n_inner": 3072, "vocab_size": 50257,
                               "n_positions": 1024}, "ids": "gpt2__ids", "seq": 8,
                    "logits_sha": sha(y.logits), "layers": layers}
    # keep the inputs of the first block and the LM head only (size); every layer's output hash and status
    keep = {layers[i]["key"] for i in (0, 1, 2, 3, len(layers) - 1)}
    for lay in layers:
        lay["out_sha"] = hashlib.sha256(arrays[lay["key"] + "__out"].tobytes()).hexdigest()
        lay["in_sha"] = hashlib.sha256(arrays[lay["key"] + "__in"].tobytes()).hexdigest()
        if lay["key"] not in keep:
            del arrays[lay["key"] + "__in"], arrays[lay["key"] + "__out"]
            lay["recorded"] = False
        else:
            lay["recorded"] = True
            if arrays[lay["key"] + "__out"].size > 100_000:      # the LM head: its output by hash only
                del arrays[lay["key"] + "__out"]
    with open(os.path.join(HERE, "torch_layers.json"), "w") as f:
        json.dump(meta, f, separators=(",", ":"))
    np.savez_compressed(os.path.join(HERE, "torch_layers.npz"), **arrays)
    print("wrote torch_layers.json / .npz", os.path.getsize(os.path.join(HERE, "torch_layers.npz")), "bytes")


if __name__ == "__main__":
    main(*sys.argv[1:])
