"""superfloat.python_b200.torch: SF layers for PyTorch on the B200 (the
reference's ``sf.torch`` surface for the chain accumulation).

>>> import superfloat.python_b200.torch as sft
>>> model = sft.convert(model, dtype="sf16")           # SF layers, run on the B200
>>> fast = torch.compile(model, backend="superfloat")  # sf:: ops retargeted to the device
>>> with torch.no_grad():
...     out = fast(x)
>>> sft.last_status()                                  # exact events per layer
"""
from __future__ import annotations

import torch

from . import _ops  # noqa: F401  (registers the sf:: custom ops)
from ._backend import GraphReport, compile_report, compile_reports, superfloat  # noqa: F401
from ._core import weight_cache  # noqa: F401
from ._modules import (ConversionReport, SFConfig, SFConv2d, SFHFConv1D, SFLinear, conversion_report, convert,
                       find_lm_heads, is_hf_conv1d)
from ._status import SFLayerStatus, capture_status, last_status, reset_status


def _bits(dtype) -> int:
    from .._array import resolve_dtype
    return resolve_dtype(dtype).bits


def quantize(t: torch.Tensor, dtype="sf16", scale=None) -> torch.Tensor:
    """Fake quantization: values on the SF grid, float storage, clipped
    straight-through gradient.  ``scale``: None (values in (-1, 1)),
    "dynamic" (max|t| / max) or a float."""
    if not isinstance(t, torch.Tensor):
        raise TypeError("sft.quantize expects a torch.Tensor")
    if not t.is_floating_point():
        t = t.to(torch.float64)
    if scale is None:
        return torch.ops.sf.quantize(t, _bits(dtype), "none", 1.0)
    if scale == "dynamic":
        return torch.ops.sf.quantize(t, _bits(dtype), "dynamic", 0.0)
    return torch.ops.sf.quantize(t, _bits(dtype), "fixed", float(scale))


def linear(x, weight, bias=None, dtype="sf16", scale="per_tensor", headroom="bound", name="linear", *,
           accumulate="chain", shift=None):
    """Functional SF linear (what SFLinear calls)."""
    return _ops.call_linear(x, weight, bias, SFConfig(_bits(dtype), scale, headroom, accumulate, shift), name)


def matmul(a, b, dtype="sf16", headroom="bound", name="matmul", *, accumulate="chain", shift=None):
    """Functional SF matmul of two activations (dynamic per-tensor scales);
    1-D operands follow torch.matmul."""
    cfg = SFConfig(_bits(dtype), "per_tensor", headroom, accumulate, shift)
    sq_a, sq_b = a.dim() == 1, b.dim() == 1
    y = _ops.call_matmul(a.unsqueeze(0) if sq_a else a, b.unsqueeze(-1) if sq_b else b, cfg, name)
    if sq_a:
        y = y.squeeze(-2)
    if sq_b:
        y = y.squeeze(-1)
    return y


__all__ = ["quantize", "linear", "matmul", "SFLinear", "SFConv2d", "SFHFConv1D", "SFConfig", "convert",
           "find_lm_heads", "is_hf_conv1d", "conversion_report", "ConversionReport", "last_status",
           "reset_status", "capture_status", "SFLayerStatus", "compile_report", "compile_reports", "GraphReport"]
