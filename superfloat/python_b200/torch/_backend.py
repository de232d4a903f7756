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

# float linear algebra that convert() did not turn into SF ops: reported as
# "not converted" (it runs in float, off the device)
_FLOAT_LINALG = frozenset({"linear", "matmul", "mm", "bmm", "conv1d", "conv2d", "conv3d", "addmm", "baddbmm",
                           "einsum", "__matmul__", "scaled_dot_product_attention"})


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


class _ReportLog:
    """Every graph report this process has produced, oldest first."""

    def __init__(self):
        self._items: list = []
        self._guard = threading.Lock()

    def add(self, rep: GraphReport) -> None:
        with self._guard:
            self._items.append(rep)

    def all(self) -> list:
        with self._guard:
            return list(self._items)


_LOG = _ReportLog()


def compile_reports() -> list:
    """The reports of every graph compiled with backend='superfloat'."""
    return _LOG.all()


def compile_report() -> GraphReport:
    """The report of the graph compiled last."""
    reps = _LOG.all()
    if not reps:
        raise ValueError("no graph has been compiled with backend='superfloat' yet")
    return reps[-1]


def _inference_only(tensors) -> None:
    """The compiled SF ops have no backward: refuse inputs that need one."""
    if not torch.is_grad_enabled():
        return
    if any(isinstance(t, torch.Tensor) and t.requires_grad for t in tensors):
        from .._errors import SFUnsupportedError
        raise SFUnsupportedError("the superfloat compile backend is inference-only; wrap the call in "
                                 "torch.no_grad(), or train with the eager layers from sft.convert")


# op -> (the function the node is retargeted to, how many leading tensor arguments it checks)
_DEVICE_IMPLS = {"linear": (linear_impl, 3), "matmul": (matmul_impl, 2), "linear_wide": (linear_wide_impl, 3),
                 "matmul_wide": (matmul_wide_impl, 2)}


def _on_device(op: str, device_name: str):
    """The node target for ``op`` on the device: the eager op's own
    implementation (so compiled == eager, bit for bit) behind the
    inference-only check."""
    impl, n_tensors = _DEVICE_IMPLS[op]

    def call(*args):
        _inference_only(args[:n_tensors])
        return impl(*args)
    call.__name__ = f"sf_{op}_on_{device_name}"
    return call


def _node_arg(node, position: int, keyword: str):
    """An argument of an FX node, given by position or by keyword."""
    return node.args[position] if position < len(node.args) else node.kwargs.get(keyword)


def _describe(gm, node) -> tuple[str, str]:
    """(short op name for the float-linear-algebra test, label for the report)."""
    if node.op == "call_module":
        mod = gm.get_submodule(node.target)
        return type(mod).__name__.lower(), f"{node.target} ({type(mod).__name__})"
    target = node.target
    label = target if isinstance(target, str) else (getattr(target, "__name__", None) or str(target))
    return label.split(".")[-1], label


@register_backend
def superfloat(gm: torch.fx.GraphModule, example_inputs, **kwargs):
    """Retarget every SF op node of ``gm`` that the default device runs at
    its width; report what runs where."""
    from .. import _config
    from .._device import get_device
    dev = get_device(_config.get("default_device"))
    report = GraphReport()
    targets = {}
    for node in gm.graph.nodes:
        if node.op not in ("call_function", "call_method", "call_module"):
            continue
        op = SF_OPS.get(str(node.target)) if node.op == "call_function" else None
        if op is not None:
            bits_at, name_at = SF_OP_ARGS[op]
            bits, layer = _node_arg(node, bits_at, "bits"), _node_arg(node, name_at, "name")
            if bits not in dev.widths_for(op):
                report.host_emulated.append((node.name, op, layer, f"sf{bits} is not supported on {dev.name}"))
                continue
            if op not in targets:
                targets[op] = _on_device(op, dev.name)
            node.target = targets[op]
            report.on_device.append((node.name, op, layer, dev.name))
            continue
        short, label = _describe(gm, node)
        (report.unconverted if short in _FLOAT_LINALG else report.cpu).append((node.name, label))
    gm.recompile()
    _LOG.add(report)
    return gm.forward
