"""Exception and warning types, the same names and bases as the reference's
(src/sf/_errors.py:14-101), so ``except sf.SFError`` and warning filters
written for the reference catch the same events here."""
from __future__ import annotations


class SFError(Exception):
    """Base of every exception this package raises."""


class SFWarning(RuntimeWarning):
    """Base of every warning this package issues."""


class SFTypeError(SFError, TypeError):
    """Bad dtype or operand type."""


class SFShapeError(SFError, ValueError):
    """Shape mismatch or bad size, caught on the host before a launch."""


class SFUnsupportedError(SFError, NotImplementedError):
    """Op or width not supported on the target."""


class SFLaunchError(SFError, RuntimeError):
    """Data larger than the target or its kernels allow."""


class SFDeviceError(SFError, RuntimeError):
    """Device fault or missing device library."""


class SFOverflowError(SFError, OverflowError):
    """A result outside +-max (the value returned is the saturated one)."""


class SFOverflowWarning(SFWarning):
    """The warn form of an overflow event."""


class SFUnderflowError(SFError, ArithmeticError):
    """The raise form of an underflow event."""


class SFUnderflowWarning(SFWarning):
    """A nonzero exact result became 0."""


class SFZeroDivisionError(SFError, ZeroDivisionError):
    """Division by an SF zero."""


class SFZeroDivisionWarning(SFWarning):
    """The warn form of a divide-by-zero event."""


class SFInvalidError(SFError, ValueError):
    """Invalid input (NaN) or domain error (sqrt of a negative)."""


class SFInvalidWarning(SFWarning):
    """The warn form of an invalid event."""


class SFDeviceOverflowWarning(SFWarning):
    """Saturation reported by a heavy op's status as an upper bound."""


class SFPreflightWarning(SFWarning):
    """The pre-flight probe suspects a heavy op saturates everywhere."""


__all__ = [
    "SFError", "SFWarning", "SFTypeError", "SFShapeError", "SFUnsupportedError", "SFLaunchError",
    "SFDeviceError", "SFOverflowError", "SFOverflowWarning", "SFUnderflowError", "SFUnderflowWarning",
    "SFZeroDivisionError", "SFZeroDivisionWarning", "SFInvalidError", "SFInvalidWarning",
    "SFDeviceOverflowWarning", "SFPreflightWarning",
]
