"""Torch custom ops in the ``sf`` namespace, the same names and signatures as
the reference's (src/sf/torch/_ops.py:184-417):

* ``sf::quantize(x, bits, mode, scale)``: fake quantization, clipped
  straight-through gradient;
* ``sf::linear(x, weight, bias, bits, wscale, headroom, name)``: the SF linear
  with the scale policy;
* ``sf::matmul(a, b, bits, headroom, name)``: the SF matmul of two
  activations;
* ``sf::linear_wide(x, weight, bias, bits, shift, name)`` and
  ``sf::matmul_wide(a, b, bits, shift, name)``: the same on the MX engine
  (``accumulate="wide"``) with the wide-mode shift rule; ``shift`` (an int)
  overrides it (src/sf/torch/_ops.py:305-365).

Each op is one opaque node in a ``torch.compile`` graph (what lets the
``superfloat`` backend find it).  Both eager execution and the compiled graph
run the op on the B200 through libsfb200; tensors on the CPU are copied to
the device and the result copied back, so a model kept on the CPU (as the
reference runs it) gets the reference's bits, and a model on the GPU never
leaves it.  Output dtype: float32 for float16 / bfloat16 / float32 inputs,
float64 for float64 (SF16 values need 16 significant bits).
"""
from __future__ import annotations

from typing import Optional

import torch

from . import _core, _wide
from ._status import SFLayerStatus, record

if hasattr(torch.ops, "sf") and hasattr(torch.ops.sf, "linear"):
    raise ImportError("another package already registered the sf:: torch ops (the reference's sf.torch?); "
                      "load one of them per process")


def out_dtype(dt: torch.dtype) -> torch.dtype:
    return torch.float64 if dt == torch.float64 else torch.float32


def _record(name, op, placement, bits, r: _core.CoreResult):
    record(SFLayerStatus(
        name=name, op=op, placement=placement, dtype=f"sf{bits}", outputs=r.outputs, saturated=r.saturated,
        exact=r.exact, underflow=r.underflow, input_underflow=r.input_underflow,
        weight_underflow=r.weight_underflow, bias_saturated=r.bias_saturated, headroom_bits=r.headroom_bits,
        act_scale=r.act_scale, accumulate=r.accumulate, shift_min=r.shift_min, shift_max=r.shift_max, h=r.h,
        redone=r.redone, flushed=r.flushed, acc_clipped=r.acc_clipped, guard_raised=r.guard_raised))


# --- implementations shared by eager and the compile backend ------------------------------

def linear_impl(x, weight, bias, bits, wscale, headroom, name):
    K, N = weight.shape[1], weight.shape[0]
    if x.shape[-1] != K:
        raise ValueError(f"sf.linear: input has {x.shape[-1]} features, weight expects {K}")
    dev = _core.target()
    lead = x.shape[:-1]
    od = out_dtype(x.dtype)
    r = _core.linear(x.reshape(-1, K), weight, bias, bits, wscale, headroom, dev, out_dtype=od)
    _record(name, "linear", dev.name, bits, r)
    return r.y.reshape(*lead, N).to(device=x.device, dtype=od)


def matmul_impl(a, b, bits, headroom, name):
    if a.dim() < 2 or b.dim() < 2:
        raise ValueError("sf.matmul expects operands with at least 2 dimensions")
    if a.shape[-1] != b.shape[-2]:
        raise ValueError(f"sf.matmul: shapes {tuple(a.shape)} and {tuple(b.shape)} are not aligned")
    dev = _core.target()
    r = _core.matmul(a, b, bits, headroom, dev)
    _record(name, "matmul", dev.name, bits, r)
    return r.y.to(device=a.device, dtype=out_dtype(torch.promote_types(a.dtype, b.dtype)))


def linear_wide_impl(x, weight, bias, bits, shift, name):
    K, N = weight.shape[1], weight.shape[0]
    if x.shape[-1] != K:
        raise ValueError(f"sf.linear: input has {x.shape[-1]} features, weight expects {K}")
    dev = _core.target()
    lead = x.shape[:-1]
    od = out_dtype(x.dtype)
    r = _wide.wide_linear(x.reshape(-1, K), weight, bias, bits, shift, dev, out_dtype=od)
    _record(name, "linear", dev.name, bits, r)
    return r.y.reshape(*lead, N).to(device=x.device, dtype=od)


def matmul_wide_impl(a, b, bits, shift, name):
    if a.dim() < 2 or b.dim() < 2:
        raise ValueError("sf.matmul expects operands with at least 2 dimensions")
    if a.shape[-1] != b.shape[-2]:
        raise ValueError(f"sf.matmul: shapes {tuple(a.shape)} and {tuple(b.shape)} are not aligned")
    dev = _core.target()
    od = out_dtype(torch.promote_types(a.dtype, b.dtype))
    r = _wide.wide_matmul(a, b, bits, shift, dev, out_dtype=od)
    _record(name, "matmul", dev.name, bits, r)
    return r.y.to(device=a.device, dtype=od)


# --- sf::quantize -------------------------------------------------------------------------

@torch.library.custom_op("sf::quantize", mutates_args=())
def quantize(x: torch.Tensor, bits: int, mode: str, scale: float) -> torch.Tensor:
    from .._array import _handle_events
    from .._format import FORMATS
    dev = _core.target()
    vals, codes, s, ev = _core.fake_quantize(x.detach().to(device=dev.torch_device, dtype=torch.float64),
                                             bits, mode, scale)
    _handle_events({k: int(v) for k, v in ev.items()}, FORMATS[bits], "quantize", max(1, codes.numel()))
    return vals.to(device=x.device, dtype=out_dtype(x.dtype))


@quantize.register_fake
def _(x, bits, mode, scale):
    return x.new_empty(x.shape, dtype=out_dtype(x.dtype))


def _quantize_setup(ctx, inputs, output):
    x, bits, mode, scale = inputs
    ctx.save_for_backward(x)
    ctx.bits, ctx.mode, ctx.scale = bits, mode, scale


def _quantize_backward(ctx, g):
    (x,) = ctx.saved_tensors
    from .._format import FORMATS
    fmt = FORMATS[ctx.bits]
    xv = x.detach().to(torch.float64)
    if ctx.mode == "dynamic":
        amax = _core.finite_absmax(xv)
        s = amax / (fmt.max_code / fmt.scale) if amax > 0 else 1.0
    elif ctx.mode == "fixed":
        s = ctx.scale
    else:
        s = 1.0
    inside = (xv / s).abs() < 1.0 - 2.0 ** -fmt.bits
    return (g * inside.to(g.dtype)).to(x.dtype), None, None, None


torch.library.register_autograd("sf::quantize", _quantize_backward, setup_context=_quantize_setup)


# --- sf::linear ---------------------------------------------------------------------------

@torch.library.custom_op("sf::linear", mutates_args=())
def linear(x: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor], bits: int,
           wscale: str, headroom: str, name: str) -> torch.Tensor:
    return linear_impl(x, weight, bias, bits, wscale, headroom, name)


@linear.register_fake
def _(x, weight, bias, bits, wscale, headroom, name):
    return x.new_empty(tuple(x.shape[:-1]) + (weight.shape[0],), dtype=out_dtype(x.dtype))


def _linear_setup(ctx, inputs, output):
    x, weight, bias, bits, wscale, headroom, name = inputs
    ctx.save_for_backward(x, weight)
    ctx.has_bias = bias is not None
    ctx.bits, ctx.wscale = bits, wscale


def _linear_backward(ctx, g):
    """Straight-through: the gradient of x @ W_q^T + b with the dequantized
    weights W_q (src/sf/torch/_ops.py:247-259)."""
    x, weight = ctx.saved_tensors
    from .._format import FORMATS
    w_q = _core.dequantize_weight(FORMATS[ctx.bits], weight.detach().to(torch.float64), ctx.wscale).to(g.dtype)
    g2 = g.reshape(-1, g.shape[-1])
    x2 = x.detach().reshape(-1, x.shape[-1]).to(g.dtype)
    grad_x = (g2 @ w_q).reshape(x.shape).to(x.dtype) if ctx.needs_input_grad[0] else None
    grad_w = (g2.T @ x2).to(weight.dtype) if ctx.needs_input_grad[1] else None
    grad_b = g2.sum(0).to(weight.dtype) if (ctx.has_bias and ctx.needs_input_grad[2]) else None
    return grad_x, grad_w, grad_b, None, None, None, None


torch.library.register_autograd("sf::linear", _linear_backward, setup_context=_linear_setup)


# --- sf::matmul ---------------------------------------------------------------------------

@torch.library.custom_op("sf::matmul", mutates_args=())
def matmul(a: torch.Tensor, b: torch.Tensor, bits: int, headroom: str, name: str) -> torch.Tensor:
    return matmul_impl(a, b, bits, headroom, name)


@matmul.register_fake
def _(a, b, bits, headroom, name):
    batch = torch.broadcast_shapes(a.shape[:-2], b.shape[:-2])
    return a.new_empty(tuple(batch) + (a.shape[-2], b.shape[-1]),
                       dtype=out_dtype(torch.promote_types(a.dtype, b.dtype)))


def _reduce_to(t, shape):
    while t.dim() > len(shape):
        t = t.sum(0)
    for i, n in enumerate(shape):
        if n == 1 and t.shape[i] != 1:
            t = t.sum(i, keepdim=True)
    return t


def _matmul_setup(ctx, inputs, output):
    a, b, bits, headroom, name = inputs
    ctx.save_for_backward(a, b)


def _matmul_backward(ctx, g):
    a, b = ctx.saved_tensors
    ad, bd = a.detach().to(g.dtype), b.detach().to(g.dtype)
    grad_a = _reduce_to(g @ bd.transpose(-1, -2), a.shape).to(a.dtype) if ctx.needs_input_grad[0] else None
    grad_b = _reduce_to(ad.transpose(-1, -2) @ g, b.shape).to(b.dtype) if ctx.needs_input_grad[1] else None
    return grad_a, grad_b, None, None, None


torch.library.register_autograd("sf::matmul", _matmul_backward, setup_context=_matmul_setup)


# --- wide mode: sf::linear_wide, sf::matmul_wide ----------------------------------------------

@torch.library.custom_op("sf::linear_wide", mutates_args=())
def linear_wide(x: torch.Tensor, weight: torch.Tensor, bias: Optional[torch.Tensor], bits: int,
                shift: Optional[int], name: str) -> torch.Tensor:
    return linear_wide_impl(x, weight, bias, bits, shift, name)


@linear_wide.register_fake
def _(x, weight, bias, bits, shift, name):
    return x.new_empty(tuple(x.shape[:-1]) + (weight.shape[0],), dtype=out_dtype(x.dtype))


def _linear_wide_setup(ctx, inputs, output):
    x, weight, bias, bits, shift, name = inputs
    ctx.save_for_backward(x, weight)
    ctx.has_bias = bias is not None
    ctx.bits = bits


def _linear_wide_backward(ctx, g):
    """Straight-through: the gradient of x @ W_q^T + b with W_q the weights as
    wide mode quantizes them, one power-of-two exponent per output channel
    (src/sf/torch/_ops.py:325-339)."""
    x, weight = ctx.saved_tensors
    from .._format import FORMATS
    fmt = FORMATS[ctx.bits]
    w = weight.detach().to(torch.float64)
    if not w.is_cuda:
        w = w.to(_core.target().torch_device)
    e = _wide.row_exponents(w)
    qw, _ = _wide.quantize_rows(fmt, w.contiguous(), e)
    w_q = (qw.to(torch.float64) * _wide.exp2(e - (fmt.bits - 1))[:, None]).to(device=g.device, dtype=g.dtype)
    g2 = g.reshape(-1, g.shape[-1])
    x2 = x.detach().reshape(-1, x.shape[-1]).to(g.dtype)
    grad_x = (g2 @ w_q).reshape(x.shape).to(x.dtype) if ctx.needs_input_grad[0] else None
    grad_w = (g2.T @ x2).to(weight.dtype) if ctx.needs_input_grad[1] else None
    grad_b = g2.sum(0).to(weight.dtype) if (ctx.has_bias and ctx.needs_input_grad[2]) else None
    return grad_x, grad_w, grad_b, None, None, None


torch.library.register_autograd("sf::linear_wide", _linear_wide_backward, setup_context=_linear_wide_setup)


@torch.library.custom_op("sf::matmul_wide", mutates_args=())
def matmul_wide(a: torch.Tensor, b: torch.Tensor, bits: int, shift: Optional[int], name: str) -> torch.Tensor:
    return matmul_wide_impl(a, b, bits, shift, name)


@matmul_wide.register_fake
def _(a, b, bits, shift, name):
    batch = torch.broadcast_shapes(a.shape[:-2], b.shape[:-2])
    return a.new_empty(tuple(batch) + (a.shape[-2], b.shape[-1]),
                       dtype=out_dtype(torch.promote_types(a.dtype, b.dtype)))


torch.library.register_autograd("sf::matmul_wide", lambda ctx, g: _matmul_backward(ctx, g)[:2] + (None, None, None),
                                setup_context=lambda ctx, inputs, output: ctx.save_for_backward(inputs[0], inputs[1]))


def call_linear(x, weight, bias, cfg, name):
    if cfg.accumulate == "wide":
        return torch.ops.sf.linear_wide(x, weight, bias, cfg.bits, cfg.shift, name)
    return torch.ops.sf.linear(x, weight, bias, cfg.bits, cfg.scale, cfg.headroom, name)


def call_matmul(a, b, cfg, name):
    if cfg.accumulate == "wide":
        return torch.ops.sf.matmul_wide(a, b, cfg.bits, cfg.shift, name)
    return torch.ops.sf.matmul(a, b, cfg.bits, cfg.headroom, name)


SF_OPS = {"sf.linear": "linear", "sf.linear.default": "linear", "sf.matmul": "matmul",
          "sf.matmul.default": "matmul", "sf.linear_wide": "linear_wide", "sf.linear_wide.default": "linear_wide",
          "sf.matmul_wide": "matmul_wide", "sf.matmul_wide.default": "matmul_wide"}
SF_OP_ARGS = {"linear": (3, 6), "matmul": (2, 4), "linear_wide": (3, 5), "matmul_wide": (2, 4)}
