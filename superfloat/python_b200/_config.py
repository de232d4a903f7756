"""Runtime knobs: sf.config (reference src/sf/_config.py:38-55) and the
accumulation mode sf.accumulate (src/sf/_accumulate.py:26-101).

Keys kept: preflight, suspect, probe, probe_size, status, offload_threshold,
default_device (the kernel-DSL keys of the reference are outside this
package).  ``default_device`` defaults to "b200".  Context-local.
"""
from __future__ import annotations

import contextvars
import functools
import inspect
from types import MappingProxyType

DEFAULTS = MappingProxyType({
    "preflight": "raise",
    "suspect": "warn",
    "probe": True,
    "probe_size": 256,
    "status": "scan",
    "offload_threshold": None,
    "default_device": "b200",
})
CHOICES = {
    "preflight": ("raise", "warn", "ignore"),
    "suspect": ("raise", "warn", "verify", "ignore"),
    "status": ("scan", "replay"),
}

_cfg = contextvars.ContextVar("sfb200_config", default=DEFAULTS)


def _validate(k, v):
    if k not in DEFAULTS:
        raise ValueError(f"unknown config key {k!r}; expected one of {tuple(DEFAULTS)}")
    if k in CHOICES and v not in CHOICES[k]:
        raise ValueError(f"{k} must be one of {CHOICES[k]}, got {v!r}")
    if k == "probe_size" and (not isinstance(v, int) or v < 1):
        raise ValueError("probe_size must be a positive int")
    if k == "offload_threshold" and v is not None and (not isinstance(v, int) or v < 0):
        raise ValueError("offload_threshold must be None or a non-negative int")


def get(key):
    return _cfg.get()[key]


def getconfig() -> dict:
    return dict(_cfg.get())


class config:
    """Set options: a plain call applies for the rest of the context, ``with``
    scopes them, a decorator applies them inside each call."""

    def __init__(self, **kw):
        for k, v in kw.items():
            _validate(k, v)
        self._kw = kw
        self._tokens = contextvars.ContextVar("sfb200_config_tokens", default=())
        self._tokens.set((self._push(),))
        self._pending = True

    def _push(self):
        return _cfg.set(MappingProxyType({**_cfg.get(), **self._kw}))

    def __enter__(self):
        if self._pending:
            self._pending = False
        else:
            self._tokens.set(self._tokens.get() + (self._push(),))
        return self

    def __exit__(self, *exc):
        stack = self._tokens.get()
        if not stack:
            raise RuntimeError("config.__exit__ without a matching __enter__")
        self._pending = False
        self._tokens.set(stack[:-1])
        _cfg.reset(stack[-1])

    def __call__(self, fn):
        if self._pending:
            self.__exit__(None, None, None)
        kw = self._kw

        @functools.wraps(fn)
        def wrap(*a, **k):
            c = config(**kw)
            try:
                return fn(*a, **k)
            finally:
                c.__exit__(None, None, None)
        return wrap


# --- accumulation mode ----------------------------------------------------------------------

MODES = ("chain", "wide")
_mode = contextvars.ContextVar("sfb200_accumulate", default="chain")


def check_mode(mode):
    if mode not in MODES:
        raise ValueError(f"accumulate must be one of {MODES}, got {mode!r}")
    return mode


def resolve_mode(mode):
    return _mode.get() if mode is None else check_mode(mode)


def getaccumulate():
    return _mode.get()


def setaccumulate(mode):
    old = _mode.get()
    _mode.set(check_mode(mode))
    return old


class accumulate:
    """Scope the accumulation mode of ``@`` / matmul / dot: "chain" (fma
    chain, the default) or "wide" (the MX engine)."""

    def __init__(self, mode):
        self._m = check_mode(mode)
        self._tokens = contextvars.ContextVar("sfb200_accumulate_tokens", default=())

    def __enter__(self):
        self._tokens.set(self._tokens.get() + (_mode.set(self._m),))
        return self

    def __exit__(self, *exc):
        stack = self._tokens.get()
        self._tokens.set(stack[:-1])
        _mode.reset(stack[-1])

    def __call__(self, fn):
        if inspect.isgeneratorfunction(fn) or inspect.isasyncgenfunction(fn):
            raise TypeError("accumulate cannot decorate a generator function")
        m = self._m

        @functools.wraps(fn)
        def wrap(*a, **k):
            with accumulate(m):
                return fn(*a, **k)
        return wrap
