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


def _head_from_output_embeddings(model, linears, embeddings) -> dict:
    get = getattr(model, "get_output_embeddings", None)
    if not callable(get):
        return {}
    try:
        head = get()
    except Exception:  # noqa: BLE001  (a model's own hook may raise)
        return {}
    if isinstance(head, nn.Module) and _linear_like(head):
        return {id(head): "LM head (the model's get_output_embeddings())"}
    return {}


def _heads_tied_to_embeddings(model, linears, embeddings) -> dict:
    def shares(w, e):
        return w is e.weight or (w is not None and w.data_ptr() == e.weight.data_ptr()
                                 and w.numel() == e.weight.numel())
    return {id(m): "LM head (weight tied to the embeddings)" for m in linears
            if any(shares(getattr(m, "weight", None), e) for e in embeddings)}


def _head_by_vocabulary(model, linears, embeddings) -> dict:
    vocab = {e.num_embeddings for e in embeddings}
    hits = [m for m in linears if (getattr(m, "out_features", None) or getattr(m, "nf", None)) in vocab]
    return {id(hits[-1]): "LM head (last layer with the vocabulary's output size)"} if hits else {}


def find_lm_heads(model: nn.Module) -> dict:
    """The LM head(s), {id(module): why}, by the first rule that finds one:
    the model's get_output_embeddings(); a linear tied to an embedding's
    weight; the last linear whose output size is an embedding's vocabulary
    (src/sf/torch/_modules.py:263-292).  The last two need an nn.Embedding."""
    linears = [m for m in model.modules() if _linear_like(m)]
    embeddings = [m for m in model.modules() if isinstance(m, nn.Embedding)]
    for rule in (_head_from_output_embeddings, _heads_tied_to_embeddings, _head_by_vocabulary):
        if rule is not _head_from_output_embeddings and not embeddings:
            return {}
        found = rule(model, linears, embeddings)
        if found:
            return found
    return {}


def _custom_forward(m, base) -> bool:
    return type(m).forward is not base.forward


# layer types with no SF form: reported as skipped, run in float
_NO_SF_FORM = (nn.Conv1d, nn.Conv3d, nn.ConvTranspose1d, nn.ConvTranspose2d, nn.ConvTranspose3d, nn.Bilinear,
               nn.LSTM, nn.GRU, nn.RNN, nn.MultiheadAttention)


def _module_names(model) -> set:
    return {n for n, _ in model.named_modules(remove_duplicate=False)}


def _unknown_names(model, names, what):
    missing = sorted(set(names) - _module_names(model))
    if missing:
        raise ValueError(f"{what}: no module named {', '.join(map(repr, missing))}")


class _Converter:
    """One pass of ``convert``: the width each layer gets, the SF layer that
    replaces it, the report.  A module reached twice (a shared submodule) is
    replaced once and the alias recorded."""

    def __init__(self, cfg, cfg16, per_layer, keep_ids, keep_names):
        self.cfg, self.cfg16 = cfg, cfg16
        self.per_layer = per_layer              # path -> SFConfig (widths=)
        self.keep_ids, self.keep_names = keep_ids, keep_names
        self.report = ConversionReport()
        self.replaced = {}                      # id(module) -> (first path, replacement or None)
        self.walked = set()

    def config_for(self, module, path) -> SFConfig:
        if path in self.per_layer:
            c = self.per_layer[path]
        elif self.cfg.bits < 16 and (id(module) in self.keep_ids or path in self.keep_names):
            self.report.kept_sf16.append((path, self.keep_ids.get(id(module)) or "named in keep_sf16"))
            c = self.cfg16
        else:
            c = self.cfg
        self.report.widths[path] = c.bits
        return c

    def _skip(self, path, kind, why):
        self.report.skipped.append((path, kind, why))

    def _make(self, module, path):
        """(SF replacement or None, whether the module is a leaf of the walk)."""
        kind = type(module).__name__
        if isinstance(module, (SFLinear, SFConv2d, SFHFConv1D)):
            self.report.converted.append((path, kind + " (already SF)"))
            return None, True
        if isinstance(module, nn.Linear):
            if _custom_forward(module, nn.Linear):
                self._skip(path, kind, f"a subclass of nn.Linear with its own forward ({kind}); runs as it was")
            elif not module.weight.is_floating_point():
                self._skip(path, kind, f"weights stored as {module.weight.dtype}")
            else:
                self.report.converted.append((path, "Linear"))
                return SFLinear.from_float(module, path, self.config_for(module, path)), True
            return None, True
        if is_hf_conv1d(module):
            if not module.weight.is_floating_point():
                self._skip(path, kind, f"weights stored as {module.weight.dtype}")
                return None, True
            self.report.converted.append((path, "Conv1D (Hugging Face)"))
            return SFHFConv1D(module, path, self.config_for(module, path)), True
        if isinstance(module, nn.Conv2d):
            ok, why = convertible_conv(module)
            if not (ok and module.weight.is_floating_point()):
                self._skip(path, "Conv2d", why or f"weights stored as {module.weight.dtype}")
                return None, True
            self.report.converted.append((path, "Conv2d"))
            return SFConv2d(module, path, self.config_for(module, path)), True
        if isinstance(module, _NO_SF_FORM):
            self._skip(path, kind, "no SF version here; runs in float")
            return None, True
        return None, False                      # a container: walk into it

    def replace(self, module, path):
        seen = self.replaced.get(id(module))
        if seen is not None:                    # met before: the same replacement, no second walk
            first, rep = seen
            if rep is not None:
                self.report.shared.append((path, first))
            return rep, True
        rep, leaf = self._make(module, path)
        self.replaced[id(module)] = (path, rep)
        return rep, leaf

    def walk(self, parent, prefix):
        if id(parent) in self.walked:
            return
        self.walked.add(id(parent))
        for name, child in list(parent._modules.items()):
            if child is None:
                continue
            path = f"{prefix}.{name}" if prefix else name
            rep, leaf = self.replace(child, path)
            if rep is not None:
                setattr(parent, name, rep)
            elif not leaf:
                self.walk(child, path)

    def run(self, model):
        rep, leaf = self.replace(model, "")
        if rep is not None:
            model = rep
        elif not leaf:
            self.walk(model, "")
        model._sf_conversion_report = self.report
        return model


def _keep_plan(model, keep_sf16, bits):
    """(LM heads by id, module names) that stay at sf16 when ``bits`` < 16."""
    if keep_sf16 == "auto":
        return (find_lm_heads(model) if bits < 16 else {}), set()
    if keep_sf16 in (False, None):
        return {}, set()
    if isinstance(keep_sf16, str) or not hasattr(keep_sf16, "__iter__"):
        raise ValueError(f"keep_sf16 must be \"auto\", False or a list of module names, got {keep_sf16!r}")
    names = set(keep_sf16)
    if bits < 16:
        _unknown_names(model, names, "keep_sf16")
    return {}, names


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
    keep_ids, keep_names = _keep_plan(model, keep_sf16, cfg.bits)
    per_layer = {}
    if widths:
        _unknown_names(model, widths, "widths")
        per_layer = {n: SFConfig(_bits_of(d), scale, headroom, accumulate, shift) for n, d in widths.items()}
    cfg16 = SFConfig(16, scale, headroom, accumulate, shift)
    return _Converter(cfg, cfg16, per_layer, keep_ids, keep_names).run(model)


def conversion_report(model: nn.Module) -> ConversionReport:
    r = getattr(model, "_sf_conversion_report", None)
    if r is None:
        raise ValueError("model was not produced by sft.convert")
    return r
