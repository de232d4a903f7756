"""Regenerate tests/golden/gpt2_64.json from the reference's sf.torch (CPU).

    SF_REFERENCE_ROOT=<reference checkout> SF_CACHE_DIR=/tmp/sfcache \
        python tests/golden/make_golden_gpt2.py

The GPT-2-small architecture (12 layers, d_model 768, 12 heads, FFN 3072,
vocab 50257; random init, torch.manual_seed(0)) converted with the
reference's ``sft.convert(model, dtype="sf16")`` (chain accumulation,
per-tensor scales, headroom "bound") and run on the CPU:

* ``seq64``: one sequence of 64 token ids (torch.Generator seed 0).  Every SF
  layer's input and output hash (float32 bytes) and ``SFLayerStatus``, and the
  logits hash.  About 3.5 minutes of the reference's host path.
* ``c_attn_8x512``: block 0's ``attn.c_attn`` (an HF Conv1D, 768 -> 2304) on
  its full-size input of the 8 x 512-token batch (torch.Generator seed 0 ids,
  so 4096 x 768 activations), i.e. one layer of the 8 x 512 forward at its
  real shape.  The input is ln_1 of the embeddings, computed by the model's
  own float modules; its hash, the output's hash and the status are kept.

Only hashes and statuses are stored (the inputs are recomputed from the
seeds by the same CPU float modules, and the test checks their hashes).
"""
from __future__ import annotations

import hashlib
import json
import os
import sys
import time

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
from _refroot import reference_root  # noqa: E402

HERE = os.path.dirname(os.path.abspath(__file__))
STATUS_KEYS = ("op", "dtype", "outputs", "saturated", "exact", "underflow", "input_underflow", "weight_underflow",
               "bias_saturated", "headroom_bits", "act_scale")
CONFIG = {"n_layer": 12, "n_embd": 768, "n_head": 12, "n_inner": 3072, "vocab_size": 50257, "n_positions": 1024}


def sha(t) -> str:
    return hashlib.sha256(t.detach().contiguous().numpy().tobytes()).hexdigest()


def block0_input(model, ids):
    """ln_1 of block 0 applied to the token + position embeddings: the input
    of block 0's c_attn, from the model's own float modules."""
    import torch
    tr = model.transformer
    pos = torch.arange(ids.shape[1]).unsqueeze(0)
    h = tr.drop(tr.wte(ids) + tr.wpe(pos))
    return tr.h[0].ln_1(h)


def main() -> None:
    ref = reference_root(sys.argv[1] if len(sys.argv) > 1 else None)
    sys.path.insert(0, os.path.join(ref, "src"))
    os.environ.setdefault("SF_CACHE_DIR", "/tmp/sf_cache_golden")
    import torch
    import sf.torch as sft          # the reference
    from transformers import GPT2Config, GPT2LMHeadModel

    torch.manual_seed(0)
    model = GPT2LMHeadModel(GPT2Config(**CONFIG)).eval()
    conv = sft.convert(model, dtype="sf16")
    out = {"config": CONFIG}

    # one layer at the 8 x 512 batch's full shape
    ids = torch.randint(0, 50257, (8, 512), generator=torch.Generator().manual_seed(0))
    with torch.no_grad():
        x = block0_input(conv, ids)
        layer = conv.transformer.h[0].attn.c_attn
        sft.reset_status()
        t0 = time.time()
        y = layer(x)
        dt = time.time() - t0
    s = sft.last_status(conv)[layer.sf_name]
    out["c_attn_8x512"] = {"name": layer.sf_name, "ids_shape": [8, 512], "in_shape": list(x.shape),
                           "in_sha": sha(x), "out_sha": sha(y), "seconds": round(dt, 1),
                           "status": {k: getattr(s, k) for k in STATUS_KEYS}}
    print(f"c_attn 8x512: {dt:.1f} s", flush=True)

    # the whole model on 64 tokens
    ids = torch.randint(0, 50257, (1, 64), generator=torch.Generator().manual_seed(0))
    seen = []
    hooks = [m.register_forward_hook(lambda mod, i, o: seen.append((mod.sf_name, type(mod).__name__,
                                                                       list(i[0].shape), sha(i[0]), sha(o))))
             for m in conv.modules() if hasattr(m, "sf_name")]
    with torch.no_grad():
        sft.reset_status()
        t0 = time.time()
        logits = conv(ids).logits
        dt = time.time() - t0
    for h in hooks:
        h.remove()
    st = sft.last_status(conv)
    layers = [{"name": n, "kind": kind, "in_shape": shp, "in_sha": i, "out_sha": o,
               "status": {k: getattr(st[n], k) for k in STATUS_KEYS}} for n, kind, shp, i, o in seen]
    out["seq64"] = {"ids_shape": [1, 64], "seconds": round(dt, 1), "logits_sha": sha(logits), "layers": layers}
    print(f"seq64 forward: {dt:.1f} s, {len(layers)} SF layers", flush=True)
    with open(os.path.join(HERE, "gpt2_64.json"), "w") as f:
        json.dump(out, f, indent=0, separators=(",", ":"))
    print("wrote gpt2_64.json")


if __name__ == "__main__":
    main()
