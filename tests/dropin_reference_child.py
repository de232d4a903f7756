"""The B200 target plugged into the reference's OWN runtime (a child process).

    python tests/dropin_reference_child.py <reference site dir> <repo> <device under test>

Imports the reference package ``sf`` from <reference site dir> (the directory
holding ``sf/``), registers ``superfloat.python_b200.B200Device`` with the
reference's ``sf.register_device`` (src/sf/_device.py:199-201), and drives
it only through the reference's public API:

* ``sf.from_codes(..., device=...)`` arrays and their operators / ``sf.fma`` /
  ``sf.div`` (the reference's ``_run_heavy`` -> ``Device.run`` path,
  src/sf/_array.py:527-591), at sf16, sf8 and sf5;
* ``sf.matmul`` in chain and wide mode, small and at a size the tensor-core
  path takes;
* a model converted by the reference's ``sft.convert`` and compiled with the
  reference's ``torch.compile(backend="superfloat")`` under
  ``sf.config(default_device=...)`` (src/sf/torch/_backend.py:135-176), and
  GPT-2-small on 8 tokens the same way.

Each result is compared with the reference's host path (codes) and with its
own flagged mock target ``atreides-flags`` (codes and ``SFStatus``, which a
sticky-flag target reports exactly), and the float outputs of the compiled
models with the reference's eager host run.  Prints one JSON line: the
checks that ran, the mismatches (empty when everything is equal) and the
device's launch count.  With <device under test> = ``atreides-flags`` the
script checks itself on a CPU-only machine.

The reference and this package both register a TorchDynamo backend named
``superfloat``, so they cannot share one interpreter: the pytest side runs
this file as a subprocess.
"""
from __future__ import annotations

import hashlib
import json
import os
import sys


def main(ref_site: str, repo: str, dut: str) -> int:
    sys.path.insert(0, ref_site)
    sys.path.insert(1, repo)
    os.environ.setdefault("SF_CACHE_DIR", os.path.join(os.environ.get("TMPDIR", "/tmp"), "sf_dropin_cache"))
    import numpy as np
    import torch
    import torch.nn as nn

    import sf                                   # the reference
    import sf.torch as sft
    from sf import _vectorized as vec
    if dut == "b200":
        from superfloat.python_b200._device import B200Device
        dev = B200Device(0)
        sf.register_device(dev)
    assert sf.get_device(dut).name == dut
    dev = sf.get_device(dut)
    launches0 = dev.launches
    checks, bad = [], []

    def same(what, a, b):
        checks.append(what)
        if not np.array_equal(np.asarray(a), np.asarray(b)):
            bad.append(what)

    def status_tuple(s):
        return None if s is None else (s.saturated, s.div0, s.invalid, s.exact, s.outputs_at_max,
                                       getattr(s, "underflow", None))

    rng = np.random.default_rng(0)
    # elementwise through the runtime's heavy-op path
    for bits in (16, 8, 5):
        dt = sf.dtypes[bits - 4]
        M = (1 << (bits - 1)) - 1
        n = 6000
        a, b, c = (rng.integers(-M, M + 1, n) for _ in range(3))
        a[:600] = rng.integers(-(M // 60) - 1, M // 60 + 2, 600)        # products that underflow
        b[:600] = rng.integers(-(M // 60) - 1, M // 60 + 2, 600)
        d = b.copy()
        d[::97] = 0                                                        # divide events
        for op in ("add", "sub", "mul", "fma", "div"):
            if dev.supported_ops is not None and op not in dev.supported_ops:
                continue                           # the mock's dry run: it has no divider
            ops = {"add": (a, b), "sub": (a, b), "mul": (a, b), "fma": (a, b, c), "div": (a, d)}[op]

            def run(device):
                xs = [sf.from_codes(np.asarray(v, dtype=np.int64), dt, device=device) for v in ops]
                with sf.errstate(all="ignore"):
                    if op == "add":
                        return xs[0] + xs[1]
                    if op == "sub":
                        return xs[0] - xs[1]
                    if op == "mul":
                        return xs[0] * xs[1]
                    if op == "fma":
                        return sf.fma(xs[0], xs[1], xs[2])
                    return sf.div(xs[0], xs[1])
            host, got = run("host"), run(dut)
            same(f"sf{bits} {op} codes vs host", got.codes, host.codes)
            if op != "div":
                flagged = run("atreides-flags")
                checks.append(f"sf{bits} {op} status vs atreides-flags")
                if status_tuple(got.status) != status_tuple(flagged.status):
                    bad.append(f"sf{bits} {op} status vs atreides-flags")
            else:
                # the flagged mock has no divider: its events come from the reference's vec.div
                _, ev = vec.div(dt._fmt, a, d)
                checks.append(f"sf{bits} div status vs vec.div events")
                st = got.status
                if st is None or st.saturated != int(ev["overflow"].sum()) or st.div0 != int(ev["divide"].sum()):
                    bad.append(f"sf{bits} div status vs vec.div events")

    # matmul, chain and wide, through sf.matmul
    for (m, k, n_) in ((37, 50, 29), (300, 1000, 260)):
        A = rng.integers(-2000, 2001, (m, k))
        B = rng.integers(-32767, 32768, (k, n_))
        for mode, kw in (("chain", {}), ("wide", {"accumulate": "wide", "shift": -2})):
            def mm(device):
                x = sf.from_codes(A, sf.sf16, device=device)
                y = sf.from_codes(B, sf.sf16, device=device)
                with sf.errstate(all="ignore"):
                    return sf.matmul(x, y, **kw)
            host, got, flagged = mm("host"), mm(dut), mm("atreides-flags")
            same(f"matmul {mode} {m}x{k}x{n_} codes vs host", got.codes, host.codes)
            checks.append(f"matmul {mode} {m}x{k}x{n_} status vs atreides-flags")
            if status_tuple(got.status) != status_tuple(flagged.status):
                bad.append(f"matmul {mode} {m}x{k}x{n_} status vs atreides-flags")

    # a converted model, eager on the host vs compiled onto the target
    torch.manual_seed(0)
    model = sft.convert(nn.Sequential(nn.Linear(64, 96), nn.GELU(), nn.Linear(96, 32)))
    x = torch.randn(20, 64) * 2
    with torch.no_grad():
        eager = model(x)
        st_host = {k: (v.saturated, v.underflow, v.act_scale) for k, v in sft.last_status(model).items()}
        torch._dynamo.reset()
        n0 = dev.launches
        with sf.config(default_device=dut):
            out = torch.compile(model, backend="superfloat")(x)
        st_dev = sft.last_status(model)
    same("compiled MLP output vs eager host", out, eager)
    checks.append("compiled MLP on the target")
    if dev.launches == n0 or any(v.placement != dut for v in st_dev.values()):
        bad.append("compiled MLP on the target")
    checks.append("compiled MLP status vs eager host")
    if {k: (v.saturated, v.underflow, v.act_scale) for k, v in st_dev.items()} != st_host:
        bad.append("compiled MLP status vs eager host")

    # GPT-2-small, 8 tokens, compiled onto the target: the logits of the reference's host run
    gold = os.path.join(repo, "tests", "golden", "torch_layers.json")
    if os.path.exists(gold):
        g = json.load(open(gold))["gpt2"]
        from transformers import GPT2Config, GPT2LMHeadModel
        torch.manual_seed(0)
        gpt = sft.convert(GPT2LMHeadModel(GPT2Config(**g["config"])).eval(), dtype="sf16")
        ids = torch.randint(0, 50257, (1, 8), generator=torch.Generator().manual_seed(0))
        torch._dynamo.reset()
        n0 = dev.launches
        with torch.no_grad(), sf.config(default_device=dut):
            logits = torch.compile(gpt, backend="superfloat")(ids).logits
        st = sft.last_status(gpt)
        checks.append("GPT-2 8 tokens compiled on the target: logits vs the reference's host run")
        if hashlib.sha256(logits.contiguous().numpy().tobytes()).hexdigest() != g["logits_sha"]:
            bad.append("GPT-2 8 tokens compiled on the target: logits vs the reference's host run")
        checks.append("GPT-2 8 tokens compiled on the target: every layer placed and statuses")
        want = {lay["name"]: lay["status"] for lay in g["layers"]}
        if dev.launches == n0 or len(st) != 49 or any(v.placement != dut for v in st.values()) or any(
                (v.saturated, v.underflow, v.act_scale) != (want[k]["saturated"], want[k]["underflow"],
                                                             want[k]["act_scale"]) for k, v in st.items()):
            bad.append("GPT-2 8 tokens compiled on the target: every layer placed and statuses")
    print(json.dumps({"device": dut, "checks": checks, "mismatches": bad, "launches": dev.launches - launches0}))
    return 0


if __name__ == "__main__":
    sys.exit(main(*sys.argv[1:4]))
