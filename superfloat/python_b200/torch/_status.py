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


class _Ledger:
    """The newest status of every SF layer, by name (all threads), plus the
    collectors that the calling context has open.  A context's collectors
    are a chain of frames held in a context variable: a frame is (its dict,
    the frame it was opened inside), so nested and concurrent captures each
    see exactly the layers run inside them."""

    def __init__(self):
        self._newest: dict = {}
        self._guard = threading.Lock()
        self._frames = contextvars.ContextVar("sfb200_layer_status_frames", default=None)

    def post(self, st: SFLayerStatus) -> None:
        with self._guard:
            self._newest[st.name] = st
        frame = self._frames.get()
        while frame is not None:
            sink, frame = frame
            sink[st.name] = st

    def open(self, sink: dict):
        return self._frames.set((sink, self._frames.get()))

    def close(self, token) -> None:
        self._frames.reset(token)

    def snapshot(self) -> dict:
        with self._guard:
            return dict(self._newest)

    def clear(self) -> None:
        with self._guard:
            self._newest.clear()


_LEDGER = _Ledger()


def record(st: SFLayerStatus) -> None:
    """Publish one layer call's status (the custom ops call this)."""
    _LEDGER.post(st)


class capture_status:
    """Collect the statuses of the SF layers run inside this context (this
    thread or task only): ``with capture_status() as st: ...`` fills the dict
    ``st``.  Used as a decorator, each call of the function collects afresh
    and the dict of the latest call is the function's ``last`` attribute."""

    def __init__(self):
        self.statuses: dict = {}
        self._open: list = []

    def __enter__(self) -> dict:
        self._open.append(_LEDGER.open(self.statuses))
        return self.statuses

    def __exit__(self, *exc) -> None:
        _LEDGER.close(self._open.pop())

    def __call__(self, fn):
        def collect():
            sink = {}
            return sink, _LEDGER.open(sink)

        if inspect.iscoroutinefunction(fn):
            async def runner(*args, **kwargs):
                sink, token = collect()
                try:
                    out = await fn(*args, **kwargs)
                finally:
                    _LEDGER.close(token)
                runner.last = sink                 # only a call that returned replaces it
                return out
        else:
            def runner(*args, **kwargs):
                sink, token = collect()
                try:
                    out = fn(*args, **kwargs)
                finally:
                    _LEDGER.close(token)
                runner.last = sink
                return out
        functools.update_wrapper(runner, fn)
        runner.last = {}
        return runner


def last_status(model=None) -> dict:
    """Status of the latest call of every SF layer, by layer name; with
    ``model``, only that model's SF layers that have run, in module order."""
    newest = _LEDGER.snapshot()
    if model is None:
        return newest
    order = (m.sf_name for m in model.modules() if hasattr(m, "sf_name"))
    return {name: newest[name] for name in order if name in newest}


def reset_status() -> None:
    """Forget every recorded status (captures already open keep theirs)."""
    _LEDGER.clear()
