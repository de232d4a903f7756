"""Per-layer status of converted models: SFLayerStatus, last_status,
capture_status, reset_status (the reference's src/sf/torch/_status.py:9-157,
same fields and meaning)."""
from __future__ import annotations

import contextvars
import functools
import inspect
import threading
from dataclasses import dataclass


@dataclass(frozen=True)
class SFLayerStatus:
    """What one SF layer call reported: outputs whose chain or bias add
    saturated (exact on the B200: sticky per-output events), outputs with a
    nonzero product truncated to 0, inputs / weights quantized to 0, bias
    values that did not fit, the headroom bits given up and the activation
    scale chosen; the wide-mode fields describe the MX-engine path."""

    name: str
    op: str
    placement: str
    dtype: str
    outputs: int
    saturated: int | None
    exact: bool
    underflow: int | None
    input_underflow: int
    weight_underflow: int
    bias_saturated: int
    headroom_bits: float
    act_scale: float = 1.0
    accumulate: str = "chain"
    shift_min: int | None = None
    shift_max: int | None = None
    h: int | None = None
    redone: int = 0
    flushed: int | None = None
    acc_clipped: int | None = None
    guard_raised: int = 0

    @property
    def ok(self):
        if self.bias_saturated:
            return False
        if self.saturated is None:
            return None
        return self.saturated == 0

    def __repr__(self):
        sat = "unknown" if self.saturated is None else str(self.saturated)
        if self.accumulate == "wide":
            fl = "unknown" if self.flushed is None else str(self.flushed)
            return (f"SFLayerStatus({self.name!r}, {self.op} wide on {self.placement}, {self.dtype}, "
                    f"shift={self.shift_min}..{self.shift_max}, h={self.h}, redone={self.redone}, "
                    f"flushed={fl}, saturated={sat})")
        return (f"SFLayerStatus({self.name!r}, {self.op} on {self.placement}, {self.dtype}, saturated={sat}, "
                f"underflow={self.underflow}, headroom_bits={self.headroom_bits:.2f})")


_lock = threading.Lock()
_last: dict = {}
_captures = contextvars.ContextVar("sfb200_status_captures", default=())


def record(st: SFLayerStatus) -> None:
    with _lock:
        _last[st.name] = st
    for sink in _captures.get():
        sink[st.name] = st


class capture_status:
    """Collect the statuses of the SF layers run inside this context (this
    thread or task only); also a decorator (the dict is then ``fn.last``)."""

    def __init__(self):
        self.statuses = {}
        self._tokens = []

    def __enter__(self):
        self._tokens.append(_captures.set(_captures.get() + (self.statuses,)))
        return self.statuses

    def __exit__(self, *exc):
        _captures.reset(self._tokens.pop())

    def __call__(self, fn):
        if inspect.iscoroutinefunction(fn):
            @functools.wraps(fn)
            async def awrap(*a, **k):
                with capture_status() as st:
                    out = await fn(*a, **k)
                awrap.last = st
                return out
            awrap.last = {}
            return awrap

        @functools.wraps(fn)
        def wrap(*a, **k):
            with capture_status() as st:
                out = fn(*a, **k)
            wrap.last = st
            return out
        wrap.last = {}
        return wrap


def last_status(model=None) -> dict:
    """Status of the latest call of every SF layer, by layer name; with
    ``model``, only its SF layers, in module order."""
    with _lock:
        snap = dict(_last)
    if model is None:
        return snap
    names = [m.sf_name for m in model.modules() if hasattr(m, "sf_name")]
    return {n: snap[n] for n in names if n in snap}


def reset_status() -> None:
    with _lock:
        _last.clear()
