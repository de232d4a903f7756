"""``torch.compile(model, backend="superfloat")``: the reference's compile
backend (src/sf/torch/_backend.py:135-176) for the B200.

TorchDynamo hands the backend FX graphs; every ``sf::linear`` /
``sf::matmul`` node whose width the target supports is retargeted to the
device implementation (the same function the eager op runs, so compiled ==
eager bit for bit); everything else runs as traced.  A coverage report is
kept per compiled graph.  The backend is inference-only, as the reference's.
"""
from __future__ import annotations

import threading
from dataclasses import dataclass, field

import torch
from torch._dynamo import register_backend

from ._ops import SF_OP_ARGS, SF_OPS, linear_impl, linear_wide_impl, matmul_impl, matmul_wide_impl

_UNCONVERTED = {"linear", "matmul", "mm", "bmm", "conv2d", "conv1d", "conv3d", "addmm", "baddbmm", "einsum",
                "__matmul__", "scaled_dot_product_attention"}


@dataclass
class GraphReport:
    on_device: list = field(default_factory=list)        # (node, op, layer name, device)
    host_emulated: list = field(default_factory=list)    # (node, op, layer name, reason)
    cpu: list = field(default_factory=list)              # (node, target)
    unconverted: list = field(default_factory=list)      # (node, target)

    @property
    def sf_ops(self) -> int:
        return len(self.on_device) + len(self.host_emulated)

    @property
    def coverage(self) -> float:
        total = self.sf_ops + len(self.unconverted)
        return len(self.on_device) / total if total else 1.0

    def __repr__(self):
        lines = [f"GraphReport: {len(self.on_device)} SF op(s) on device, {len(self.host_emulated)} host-emulated, "
                 f"{len(self.unconverted)} float linear algebra op(s) not converted, {len(self.cpu)} other op(s) "
                 f"on CPU; linear-algebra coverage {self.coverage:.0%}"]
        lines += [f"  device  {n}: sf.{op} {name!r} on {d}" for n, op, name, d in self.on_device]
        lines += [f"  host    {n}: sf.{op} {name!r} ({why})" for n, op, name, why in self.host_emulated]
        lines += [f"  float   {n}: {t} (not converted; use sft.convert)" for n, t in self.unconverted]
        lines += [f"  cpu     {n}: {t}" for n, t in self.cpu]
        return "\n".join(lines)


_lock = threading.Lock()
_reports: list = []


def compile_reports() -> list:
    with _lock:
        return list(_reports)


def compile_report() -> GraphReport:
    with _lock:
        if not _reports:
            raise ValueError("no graph has been compiled with backend='superfloat' yet")
        return _reports[-1]


def _require_no_grad(*tensors):
    if torch.is_grad_enabled() and any(isinstance(t, torch.Tensor) and t.requires_grad for t in tensors):
        from .._errors import SFUnsupportedError
        raise SFUnsupportedError("the superfloat compile backend is inference-only; wrap the call in "
                                 "torch.no_grad(), or train with the eager layers from sft.convert")


def _device_linear(device):
    def run(x, weight, bias, bits, wscale, headroom, name):
        _require_no_grad(x, weight, bias)
        return linear_impl(x, weight, bias, bits, wscale, headroom, name)
    run.__name__ = f"sf_linear_on_{device}"
    return run


def _device_matmul(device):
    def run(a, b, bits, headroom, name):
        _require_no_grad(a, b)
        return matmul_impl(a, b, bits, headroom, name)
    run.__name__ = f"sf_matmul_on_{device}"
    return run


def _device_linear_wide(device):
    def run(x, weight, bias, bits, shift, name):
        _require_no_grad(x, weight, bias)
        return linear_wide_impl(x, weight, bias, bits, shift, name)
    run.__name__ = f"sf_linear_wide_on_{device}"
    return run


def _device_matmul_wide(device):
    def run(a, b, bits, shift, name):
        _require_no_grad(a, b)
        return matmul_wide_impl(a, b, bits, shift, name)
    run.__name__ = f"sf_matmul_wide_on_{device}"
    return run


def _arg(node, i, key):
    return node.args[i] if len(node.args) > i else node.kwargs.get(key)


def _target_name(node):
    t = node.target
    return t if isinstance(t, str) else (getattr(t, "__name__", None) or str(t))


@register_backend
def superfloat(gm: torch.fx.GraphModule, example_inputs, **kwargs):
    from .. import _config
    from .._device import get_device
    dev = get_device(_config.get("default_device"))
    report = GraphReport()
    impl = {"linear": _device_linear(dev.name), "matmul": _device_matmul(dev.name),
            "linear_wide": _device_linear_wide(dev.name), "matmul_wide": _device_matmul_wide(dev.name)}
    for node in gm.graph.nodes:
        if node.op not in ("call_function", "call_method", "call_module"):
            continue
        name = _target_name(node)
        if node.op == "call_function" and str(node.target) in SF_OPS:
            op = SF_OPS[str(node.target)]
            ib, iname = SF_OP_ARGS[op]
            bits, layer = _arg(node, ib, "bits"), _arg(node, iname, "name")
            if bits in dev.widths_for(op):
                node.target = impl[op]
                report.on_device.append((node.name, op, layer, dev.name))
            else:
                report.host_emulated.append((node.name, op, layer, f"sf{bits} is not supported on {dev.name}"))
            continue
        short = name.split(".")[-1]
        if node.op == "call_module":
            sub = gm.get_submodule(node.target)
            short = type(sub).__name__.lower()
            name = f"{node.target} ({type(sub).__name__})"
        if short in _UNCONVERTED:
            report.unconverted.append((node.name, name))
        else:
            report.cpu.append((node.name, name))
    gm.recompile()
    with _lock:
        _reports.append(report)
    return gm.forward
