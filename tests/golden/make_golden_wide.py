"""Regenerate tests/golden/wide_layers.{json,npz} from the reference's wide
sft path (CPU).

    SF_CACHE_DIR=/tmp/sfcache python tests/golden/make_golden_wide.py [reference_root]

Three parts:

1. the reference's own golden cases for the wide linear
   (spec/golden/wide/sft_wide.json, "linear"), re-emitted: x, w, b, y and
   every status field;
2. runs of ``sf.torch._core.wide_linear`` (src/sf/torch/_core.py:569-600) on
   seeded float64 inputs chosen so that every event of the wide rule fires
   somewhere: the accumulator guard raising token exponents, outputs redone
   at the l2 exponent, bias codes clamped, POP flushes, an explicit shift,
   zero rows / columns, sf16 / sf12 / sf8 / sf4 and both MX chips;
3. GPT-2-small (12 layers, d_model 768, FFN 3072, vocab 50257; random init,
   torch.manual_seed(0)) converted with ``accumulate="wide"`` and
   ``attention=False`` (scaled-dot-product attention stays in float) on one
   sequence of 8 token ids: every SF layer's status, its output hash, the inputs and
   outputs of the first block's layers, and the logits hash.
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
STATUS_KEYS = ("saturated", "exact", "underflow", "input_underflow", "weight_underflow", "bias_saturated",
               "headroom_bits", "outputs", "act_scale", "accumulate", "shift_min", "shift_max", "h", "redone",
               "flushed", "acc_clipped", "guard_raised")


def _status(r) -> dict:
    return {k: getattr(r, k) for k in STATUS_KEYS}


def seeded_cases(rng):
    """(tag, bits, mx, shift, x, w, b) with every wide event represented."""
    out = []
    for bits in (16, 12, 8, 4):
        x = rng.standard_normal((9, 40))
        w = rng.standard_normal((13, 40)) * 0.02
        b = rng.standard_normal(13) * 0.01
        out.append((f"typical_sf{bits}", bits, None, None, x, w, b))
    x = rng.standard_normal((6, 64))
    out.append(("aligned_redo_sf16", 16, None, None, x, x.copy() * 0.5, None))          # outputs at the l2 bound
    x = np.ones((4, 4096)) * 3.0
    x[1] *= -1.0
    out.append(("guard_sf16", 16, None, None, x, np.ones((5, 4096)) * 0.7, None))       # the guard raises
    out.append(("guard_v481_sf16", 16, "v4.8.1", None, rng.standard_normal((5, 300)) * 4,
                rng.standard_normal((7, 300)), rng.standard_normal(7)))
    x = rng.standard_normal((5, 32))
    w = rng.standard_normal((7, 32)) * 0.05
    b = np.array([40.0, -1e3, 0.0, 1e-9, 3.0, -2.5e-4, 7e5])
    out.append(("bias_big_sf16", 16, None, None, x, w, b))                              # bias clamps / redos
    out.append(("bias_big_sf8", 8, None, None, x, w, b))
    out.append(("shift_fixed_sf16", 16, None, -2, x, w, rng.standard_normal(7)))        # an explicit shift
    out.append(("shift_fixed_sf12", 12, None, 5, x, w, None))
    K = 64
    x = np.ones((3, K))
    w = np.tile(np.where(np.arange(K) % 2 == 0, 1.0, -1.0), (4, 1))
    w[:, 0] += 2.0 ** -14                                                               # totals far below l2: flushes
    w[2, 1] -= 2.0 ** -9
    out.append(("flush_sf16", 16, None, None, x, w, None))
    out.append(("flush_sf8", 8, None, None, x, w, None))
    x = rng.standard_normal((5, 24))
    x[2] = 0.0
    w = rng.standard_normal((6, 24))
    w[3] = 0.0
    b = rng.standard_normal(6)
    b[1] = 0.0
    out.append(("zeros_sf16", 16, None, None, x, w, b))
    x = rng.standard_normal((33, 257)) * np.logspace(-3, 3, 257)
    w = rng.standard_normal((19, 257)) * 0.05
    out.append(("ragged_sf16", 16, None, None, x, w, rng.standard_normal(19) * 0.1))
    out.append(("ragged_v481_sf12", 12, "v4.8.1", None, x, w, None))
    return out


def main(ref: str | None = None) -> None:
    ref = reference_root(ref)
    sys.path.insert(0, os.path.join(ref, "src"))
    os.environ.setdefault("SF_CACHE_DIR", "/tmp/sf_cache_golden")
    import torch
    import sf.torch as sft                       # the reference
    from sf.torch import _core

    arrays, meta = {}, {"source": "reference sf v0.16.0, sf.torch wide mode", "spec": [], "runs": []}

    spec = json.load(open(os.path.join(ref, "spec", "golden", "wide", "sft_wide.json")))
    for i, c in enumerate(spec["linear"]):
        key = f"spec{i}"
        for name in ("x", "w", "b", "y"):
            if c.get(name) is not None:
                arrays[f"{key}__{name}"] = np.asarray(c[name], dtype=np.float64)
        meta["spec"].append({"key": key, "what": c["what"], "bits": c["bits"], "has_bias": c.get("b") is not None,
                             "status": c["status"]})

    rng = np.random.default_rng(2026)
    fired = dict.fromkeys(("guard_raised", "redone", "bias_saturated", "flushed", "saturated"), 0)
    for tag, bits, mx, shift, x, w, b in seeded_cases(rng):
        r = _core.wide_linear(x, w, b, bits, shift, _core.HostRunner(), mx)
        for name, arr in (("x", x), ("w", w), ("b", b), ("y", r.y)):
            if arr is not None:
                arrays[f"{tag}__{name}"] = np.asarray(arr, dtype=np.float64)
        st = _status(r)
        for k in fired:
            fired[k] += int(st[k] or 0)
        meta["runs"].append({"key": tag, "bits": bits, "mx": mx, "shift": shift, "has_bias": b is not None,
                             "status": st})
        print(tag, {k: st[k] for k in ("redone", "guard_raised", "bias_saturated", "flushed", "saturated")})
    assert all(fired.values()), fired

    from transformers import GPT2Config, GPT2LMHeadModel
    torch.manual_seed(0)
    cfg = GPT2Config(n_layer=12, n_embd=768, n_head=12, n_inner=3072, vocab_size=50257, n_positions=1024)
    gpt = GPT2LMHeadModel(cfg).eval()
    conv = sft.convert(gpt, dtype="sf16", accumulate="wide", attention=False)
    ids = torch.randint(0, 50257, (1, 8), generator=torch.Generator().manual_seed(0))
    recs = []
    hooks = [m.register_forward_hook(lambda mod, inp, out: recs.append((mod.sf_name, inp[0].detach().clone(),
                                                                        out.detach().clone())))
             for _, m in conv.named_modules() if hasattr(m, "sf_name")]
    sft.reset_status()
    with torch.no_grad():
        y = conv(ids)
    for h in hooks:
        h.remove()
    st = sft.last_status(conv)
    layers = []
    for i, (name, xin, yout) in enumerate(recs):
        s = st[name]
        lay = {"name": name, "key": f"gpt2__{i}", "in_shape": list(xin.shape),
               "in_sha": hashlib.sha256(xin.contiguous().numpy().tobytes()).hexdigest(),
               "out_sha": hashlib.sha256(yout.contiguous().numpy().tobytes()).hexdigest(),
               "status": {k: getattr(s, k) for k in ("op", "dtype") + STATUS_KEYS}}
        if i < 4:                                  # the first block's layers, in and out
            arrays[lay["key"] + "__in"] = xin.numpy()
            arrays[lay["key"] + "__out"] = yout.numpy()
            lay["recorded"] = True
        layers.append(lay)
    arrays["gpt2__ids"] = ids.numpy()
    meta["gpt2"] = {"ids": "gpt2__ids", "seq": 8, "layers": layers,
                    "logits_sha": hashlib.sha256(y.logits.contiguous().numpy().tobytes()).hexdigest()}
    with open(os.path.join(HERE, "wide_layers.json"), "w") as f:
        json.dump(meta, f, indent=0)
    np.savez_compressed(os.path.join(HERE, "wide_layers.npz"), **arrays)
    print("wrote wide_layers.json / .npz", os.path.getsize(os.path.join(HERE, "wide_layers.npz")), "bytes")


if __name__ == "__main__":
    main(*sys.argv[1:])
