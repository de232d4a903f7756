"""Numeric error policy: errstate / seterr / geterr.

Same keys, values and defaults as the reference (src/sf/_errstate.py:22-29):
over=raise, under=warn, divide=raise, invalid=raise.  The value an op returns
is always the saturated / truncated one; the policy only decides whether the
host also raises or warns.  Context-local (contextvars), so threads and
asyncio tasks each see their own policy.
"""
from __future__ import annotations

import contextvars
import functools
import inspect
import os
import sys
import warnings
from types import MappingProxyType

from . import _errors

KEYS = ("over", "under", "divide", "invalid")
VALUES = ("raise", "warn", "ignore")
DEFAULTS = MappingProxyType({"over": "raise", "under": "warn", "divide": "raise", "invalid": "raise"})

_policy = contextvars.ContextVar("sfb200_errstate", default=DEFAULTS)

EVENTS = {
    "overflow": ("over", _errors.SFOverflowError, _errors.SFOverflowWarning),
    "underflow": ("under", _errors.SFUnderflowError, _errors.SFUnderflowWarning),
    "divide": ("divide", _errors.SFZeroDivisionError, _errors.SFZeroDivisionWarning),
    "invalid": ("invalid", _errors.SFInvalidError, _errors.SFInvalidWarning),
}


def _validate(key, value):
    if key not in KEYS:
        raise ValueError(f"unknown errstate key {key!r}; expected one of {KEYS}")
    if value is not None and value not in VALUES:
        raise ValueError(f"errstate value for {key!r} must be one of {VALUES}, got {value!r}")


def _merged(base, all_, kw):
    new = dict(base)
    if all_ is not None:
        new.update({k: all_ for k in KEYS})
    new.update({k: v for k, v in kw.items() if v is not None})
    return MappingProxyType(new)


def geterr() -> dict:
    return dict(_policy.get())


def seterr(all=None, **kw) -> dict:
    for k, v in kw.items():
        _validate(k, v)
    if all is not None:
        _validate("over", all)
    old = geterr()
    _policy.set(_merged(old, all, kw))
    return old


class errstate:
    """Scope a policy change; a context manager or a decorator."""

    def __init__(self, all=None, **kw):
        for k, v in kw.items():
            _validate(k, v)
        if all is not None:
            _validate("over", all)
        self._all, self._kw = all, kw
        self._tokens = contextvars.ContextVar("sfb200_errstate_tokens", default=())

    def __enter__(self):
        tok = _policy.set(_merged(_policy.get(), self._all, self._kw))
        self._tokens.set(self._tokens.get() + (tok,))
        return self

    def __exit__(self, *exc):
        stack = self._tokens.get()
        if not stack:
            raise RuntimeError("errstate.__exit__ without a matching __enter__")
        self._tokens.set(stack[:-1])
        _policy.reset(stack[-1])

    def __call__(self, fn):
        if inspect.isgeneratorfunction(fn) or inspect.isasyncgenfunction(fn):
            raise TypeError("errstate cannot decorate a generator function")
        all_, kw = self._all, self._kw
        if inspect.iscoroutinefunction(fn):
            @functools.wraps(fn)
            async def awrap(*a, **k):
                with errstate(all_, **kw):
                    return await fn(*a, **k)
            return awrap

        @functools.wraps(fn)
        def wrap(*a, **k):
            with errstate(all_, **kw):
                return fn(*a, **k)
        return wrap


_PKG = os.path.dirname(os.path.abspath(__file__))


def user_stacklevel() -> int:
    """Stack level of the first frame outside this package, so a warning
    points at the user's line."""
    level, f = 1, sys._getframe(1)
    while f is not None:
        if not os.path.abspath(f.f_code.co_filename).startswith(_PKG):
            return level
        f, level = f.f_back, level + 1
    return level


def handle(event, message: str) -> None:
    """Apply the policy to one event: raise, warn or nothing."""
    if event is None:
        return
    key, err, warn = EVENTS[event]
    action = _policy.get()[key]
    if action == "raise":
        raise err(message)
    if action == "warn":
        warnings.warn(message, warn, stacklevel=user_stacklevel())
