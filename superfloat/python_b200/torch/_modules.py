"""SF layers and model conversion: SFConfig, SFLinear, SFHFConv1D, SFConv2d,
convert, ConversionReport, find_lm_heads (the reference's
src/sf/torch/_modules.py:18-537, chain accumulation).

``convert`` swaps ``nn.Linear``, ``nn.Conv2d`` (groups=1, zero padding) and
Hugging Face's ``Conv1D`` (GPT-2) for SF layers that keep the source layer's
own parameter objects; each SF layer's forward is one ``sf::linear`` op run by
libsfb200.  Layers it cannot convert are listed in the report with the
reason and run as they were.
"""
from __future__ import annotations

import copy
from dataclasses import dataclass, field

import torch.nn as nn
import torch.nn.functional as F

from . import _core
from ._ops import call_linear


def _bits_of(dtype) -> int:
    from .._array import resolve_dtype
    return resolve_dtype(dtype).bits


@dataclass
class SFConfig:
    """How an SF layer computes: width, weight scale ("per_tensor" |
    "per_channel"), headroom ("bound": no saturation, provable | "none")."""

    bits: int = 16
    scale: str = "per_tensor"
    headroom: str = "bound"
    accumulate: str = "chain"
    shift: int | None = None

    def __post_init__(self):
        _core.check_args(self.bits, self.scale, self.headroom, self.accumulate)
        if self.shift is not None:
            if self.accumulate != "wide":
                raise ValueError("shift= only applies to accumulate=\"wide\"")
            if isinstance(self.shift, bool) or not isinstance(self.shift, int):
                raise TypeError(f"shift must be an int, got {type(self.shift).__name__}")
            if not -32 <= self.shift <= 31:
                raise ValueError(f"shift must be between -32 and 31, got {self.shift}")

    @property
    def dtype_name(self) -> str:
        return f"sf{self.bits}"

    def describe(self) -> str:
        if self.accumulate == "wide":
            return f"dtype={self.dtype_name}, accumulate=wide" + ("" if self.shift is None else f", shift={self.shift}")
        return f"dtype={self.dtype_name}, scale={self.scale}, headroom={self.headroom}"


class SFLinear(nn.Module):
    """``nn.Linear`` with SF arithmetic: the float parameters stay (training
    works through the straight-through gradient); every forward quantizes and
    runs the SF chain on the B200."""

    def __init__(self, in_features, out_features, bias=True, *, dtype="sf16", scale="per_tensor",
                 headroom="bound", accumulate="chain", shift=None, name="", device=None, param_dtype=None):
        super().__init__()
        self.in_features, self.out_features = in_features, out_features
        self.sf = SFConfig(_bits_of(dtype), scale, headroom, accumulate, shift)
        self.sf_name = name or f"linear_{id(self):x}"
        ref = nn.Linear(in_features, out_features, bias, device=device, dtype=param_dtype)
        self.weight = ref.weight
        self.bias = ref.bias

    @classmethod
    def from_float(cls, m: nn.Linear, name: str, cfg: SFConfig) -> "SFLinear":
        """Wrap ``m``'s own parameter objects (an optimizer built before the
        conversion keeps working) and its training state."""
        new = cls.__new__(cls)
        nn.Module.__init__(new)
        new.in_features, new.out_features = m.in_features, m.out_features
        new.sf = cfg
        new.sf_name = name or f"linear_{id(new):x}"
        new.weight = m.weight
        new.bias = m.bias
        new.train(m.training)
        return new

    def forward(self, x):
        return call_linear(x, self.weight, self.bias, self.sf, self.sf_name)

    def extra_repr(self):
        return (f"in_features={self.in_features}, out_features={self.out_features}, "
                f"bias={self.bias is not None}, {self.sf.describe()}, name={self.sf_name!r}")


def is_hf_conv1d(m: nn.Module) -> bool:
    """Hugging Face's ``Conv1D``: a linear layer whose weight is stored
    ``(in, out)``, recognised by name and attributes (transformers is never
    imported)."""
    w = getattr(m, "weight", None)
    return (type(m).__name__ == "Conv1D" and isinstance(getattr(m, "nf", None), int)
            and isinstance(getattr(m, "nx", None), int) and w is not None and hasattr(w, "shape")
            and tuple(w.shape) == (m.nx, m.nf))


class SFHFConv1D(nn.Module):
    """Hugging Face ``Conv1D`` with SF arithmetic: a linear on ``weight.t()``;
    the weight keeps its ``(in, out)`` layout and is the source's parameter."""

    def __init__(self, conv: nn.Module, name: str, cfg: SFConfig):
        super().__init__()
        if not is_hf_conv1d(conv):
            raise ValueError("not a Hugging Face Conv1D")
        self.nf, self.nx = conv.nf, conv.nx
        self.sf = cfg
        self.sf_name = name
        self.weight = conv.weight
        self.bias = conv.bias
        self.train(conv.training)

    def forward(self, x):
        return call_linear(x, self.weight.t(), self.bias, self.sf, self.sf_name)

    def extra_repr(self):
        return f"nf={self.nf}, nx={self.nx}, {self.sf.describe()}, name={self.sf_name!r}"


def _pair(v):
    return tuple(v) if isinstance(v, (tuple, list)) else (v, v)


def convertible_conv(c: nn.Conv2d):
    if c.groups != 1:
        return False, f"groups={c.groups} (only groups=1 is converted)"
    if c.padding_mode != "zeros":
        return False, f"padding_mode={c.padding_mode!r} (only 'zeros' is converted)"
    if isinstance(c.padding, str):
        return False, f"padding={c.padding!r} (only explicit integer padding is converted)"
    return True, ""


class SFConv2d(nn.Module):
    """``nn.Conv2d`` as unfold (data movement) + SF linear (the reduction)."""

    def __init__(self, conv: nn.Conv2d, name: str, cfg: SFConfig):
        super().__init__()
        ok, why = convertible_conv(conv)
        if not ok:
            raise ValueError(why)
        self.in_channels, self.out_channels = conv.in_channels, conv.out_channels
        self.kernel_size = _pair(conv.kernel_size)
        self.stride, self.padding, self.dilation = _pair(conv.stride), _pair(conv.padding), _pair(conv.dilation)
        self.sf = cfg
        self.sf_name = name
        self.weight = conv.weight
        self.bias = conv.bias
        self.train(conv.training)

    def forward(self, x):
        n, _, h, w = x.shape
        kh, kw = self.kernel_size
        cols = F.unfold(x, (kh, kw), dilation=self.dilation, padding=self.padding, stride=self.stride)
        oh = (h + 2 * self.padding[0] - self.dilation[0] * (kh - 1) - 1) // self.stride[0] + 1
        ow = (w + 2 * self.padding[1] - self.dilation[1] * (kw - 1) - 1) // self.stride[1] + 1
        y = call_linear(cols.transpose(1, 2), self.weight.reshape(self.out_channels, -1), self.bias, self.sf,
                        self.sf_name)
        return y.transpose(1, 2).reshape(n, self.out_channels, oh, ow)

    def extra_repr(self):
        return (f"{self.in_channels}, {self.out_channels}, kernel_size={self.kernel_size}, stride={self.stride}, "
                f"padding={self.padding}, {self.sf.describe()}, name={self.sf_name!r}")


@dataclass
class ConversionReport:
    converted: list = field(default_factory=list)     # (name, kind)
    skipped: list = field(default_factory=list)       # (name, kind, reason)
    shared: list = field(default_factory=list)        # (alias name, converted name)
    kept_sf16: list = field(default_factory=list)     # (name, why)
    attention: str = "float (not converted)"
    widths: dict = field(default_factory=dict)        # name -> bits

    def __repr__(self):
        lines = [f"ConversionReport: {len(self.converted)} converted, {len(self.skipped)} skipped"
                 + (f", {len(self.shared)} shared alias(es)" if self.shared else "")
                 + (f", {len(self.kept_sf16)} kept at sf16" if self.kept_sf16 else "")]
        if self.widths:
            per = {}
            for b in self.widths.values():
                per[b] = per.get(b, 0) + 1
            lines += ["  widths: " + ", ".join(f"sf{b} x {k}" for b, k in sorted(per.items()))]
        lines += [f"  + {n} ({k})" for n, k in self.converted]
        lines += [f"  ^ {n} kept at sf16: {w}" for n, w in self.kept_sf16]
        lines += [f"  attention: {self.attention}"]
        lines += [f"  = {a} is {n} (shared module, converted once)" for a, n in self.shared]
        lines += [f"  - {n} ({k}): {r}" for n, k, r in self.skipped]
        return "\n".join(lines)


def _linear_like(m):
    return isinstance(m, (nn.Linear, SFLinear, SFHFConv1D)) or is_hf_conv1d(m)


def find_lm_heads(model: nn.Module) -> dict:
    """The LM head(s), {id(module): why}: the model's get_output_embeddings();
    else a linear tied to an embedding's weight; else the last linear whose
    output size is an embedding's vocabulary (src/sf/torch/_modules.py:263-292)."""
    get = getattr(model, "get_output_embeddings", None)
    if callable(get):
        try:
            head = get()
        except Exception:  # noqa: BLE001  (a model's own hook may raise)
            head = None
        if isinstance(head, nn.Module) and _linear_like(head):
            return {id(head): "LM head (the model's get_output_embeddings())"}
    embs = [m for m in model.modules() if isinstance(m, nn.Embedding)]
    if not embs:
        return {}
    lins = [m for m in model.modules() if _linear_like(m)]
    tied = {}
    for m in lins:
        w = getattr(m, "weight", None)
        for e in embs:
            if w is e.weight or (w is not None and w.data_ptr() == e.weight.data_ptr()
                                 and w.numel() == e.weight.numel()):
                tied[id(m)] = "LM head (weight tied to the embeddings)"
    if tied:
        return tied
    vocab = {e.num_embeddings for e in embs}
    last = [m for m in lins if (getattr(m, "out_features", None) or getattr(m, "nf", None)) in vocab]
    return {id(last[-1]): "LM head (last layer with the vocabulary's output size)"} if last else {}


def _custom_forward(m, base) -> bool:
    return type(m).forward is not base.forward


def convert(model: nn.Module, dtype="sf16", scale: str = "per_tensor", headroom: str = "bound",
            inplace: bool = False, *, accumulate: str = "chain", shift=None, calibration: str = "heuristic",
            keep_sf16="auto", attention="auto", nonlinear: str = "float",
            widths: dict | None = None) -> nn.Module:
    """Swap ``nn.Linear``, ``nn.Conv2d`` and Hugging Face ``Conv1D`` for SF
    layers (src/sf/torch/_modules.py:295-537).  ``keep_sf16`` ("auto": the LM
    head; False; or module names) keeps layers at sf16 when ``dtype`` is
    narrower; ``widths`` ({name: dtype}) gives layers their own width."""
    if calibration not in ("heuristic",):
        raise ValueError(f"calibration must be 'heuristic', got {calibration!r}")
    if attention not in ("auto", False, None):
        raise ValueError(f"attention must be \"auto\" or False, got {attention!r}")
    if nonlinear != "float":
        from .._errors import SFUnsupportedError
        raise SFUnsupportedError("nonlinear must be \"float\" here: the integer non-linear ops are not built")
    if accumulate == "wide" and attention == "auto":
        from .._errors import SFUnsupportedError
        raise SFUnsupportedError("accumulate=\"wide\" with attention=\"auto\" runs scaled-dot-product attention "
                                 "on the MX engine, which is not built here; pass attention=False to keep "
                                 "attention in float (the layers still run wide)")
    cfg = SFConfig(_bits_of(dtype), scale, headroom, accumulate, shift)
    if not inplace:
        model = copy.deepcopy(model)
    report = ConversionReport()
    cfg16 = SFConfig(16, scale, headroom, accumulate, shift)
    keep_ids, keep_names = {}, set()
    if keep_sf16 == "auto":
        if cfg.bits < 16:
            keep_ids = find_lm_heads(model)
    elif keep_sf16 in (False, None):
        pass
    elif isinstance(keep_sf16, str) or not hasattr(keep_sf16, "__iter__"):
        raise ValueError(f"keep_sf16 must be \"auto\", False or a list of module names, got {keep_sf16!r}")
    else:
        keep_names = set(keep_sf16)
        if cfg.bits < 16:
            known = {n for n, _ in model.named_modules(remove_duplicate=False)}
            missing = sorted(keep_names - known)
            if missing:
                raise ValueError(f"keep_sf16: no module named {', '.join(map(repr, missing))}")
    per_layer = {}
    if widths:
        known = {n for n, _ in model.named_modules(remove_duplicate=False)}
        missing = sorted(set(widths) - known)
        if missing:
            raise ValueError(f"widths: no module named {', '.join(map(repr, missing))}")
        per_layer = {n: SFConfig(_bits_of(d), scale, headroom, accumulate, shift) for n, d in widths.items()}

    def cfg_for(child, full):
        if full in per_layer:
            c = per_layer[full]
        elif cfg.bits >= 16:
            c = cfg
        else:
            why = keep_ids.get(id(child)) or ("named in keep_sf16" if full in keep_names else None)
            if why is None:
                c = cfg
            else:
                report.kept_sf16.append((full, why))
                c = cfg16
        report.widths[full] = c.bits
        return c

    done, seen = {}, set()

    def replacement(child, full):
        key = id(child)
        if key in done:
            name, rep = done[key]
            if rep is not None:
                report.shared.append((full, name))
            return rep, True
        rep = None
        if isinstance(child, (SFLinear, SFConv2d, SFHFConv1D)):
            report.converted.append((full, type(child).__name__ + " (already SF)"))
        elif isinstance(child, nn.Linear):
            if _custom_forward(child, nn.Linear):
                report.skipped.append((full, type(child).__name__, f"a subclass of nn.Linear with its own forward "
                                       f"({type(child).__name__}); runs as it was"))
            elif not child.weight.is_floating_point():
                report.skipped.append((full, type(child).__name__, f"weights stored as {child.weight.dtype}"))
            else:
                rep = SFLinear.from_float(child, full, cfg_for(child, full))
                report.converted.append((full, "Linear"))
        elif is_hf_conv1d(child):
            if child.weight.is_floating_point():
                rep = SFHFConv1D(child, full, cfg_for(child, full))
                report.converted.append((full, "Conv1D (Hugging Face)"))
            else:
                report.skipped.append((full, type(child).__name__, f"weights stored as {child.weight.dtype}"))
        elif isinstance(child, nn.Conv2d):
            ok, why = convertible_conv(child)
            if ok and child.weight.is_floating_point():
                rep = SFConv2d(child, full, cfg_for(child, full))
                report.converted.append((full, "Conv2d"))
            else:
                report.skipped.append((full, "Conv2d", why or f"weights stored as {child.weight.dtype}"))
        elif isinstance(child, (nn.Conv1d, nn.Conv3d, nn.ConvTranspose1d, nn.ConvTranspose2d, nn.ConvTranspose3d,
                                nn.Bilinear, nn.LSTM, nn.GRU, nn.RNN, nn.MultiheadAttention)):
            report.skipped.append((full, type(child).__name__, "no SF version here; runs in float"))
        else:
            done[key] = (full, None)
            return None, False
        done[key] = (full, rep)
        return rep, True

    def visit(parent, prefix):
        if id(parent) in seen:
            return
        seen.add(id(parent))
        for child_name, child in list(parent._modules.items()):
            if child is None:
                continue
            full = f"{prefix}.{child_name}" if prefix else child_name
            rep, leaf = replacement(child, full)
            if rep is not None:
                setattr(parent, child_name, rep)
            elif not leaf:
                visit(child, full)

    rep, leaf = replacement(model, "")
    if rep is not None:
        model = rep
    elif not leaf:
        visit(model, "")
    model._sf_conversion_report = report
    return model


def conversion_report(model: nn.Module) -> ConversionReport:
    r = getattr(model, "_sf_conversion_report", None)
    if r is None:
        raise ValueError("model was not produced by sft.convert")
    return r
