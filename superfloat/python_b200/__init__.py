"""superfloat.python_b200: the sf hot path on B200 (sm_100a).

Bit-exact sf4..sf16 saturating fixed-point arithmetic - elementwise ops with
overflow / underflow / divide / invalid status, the chain and wide (MX
engine) matmuls, and the linear layers of ``sft.convert`` - run by
hand-written CUDA kernels in ``libsfb200.so`` behind the reference's
``Device`` plug-in interface.

    import superfloat.python_b200 as sf
    h = sf.asarray(x, dtype=sf.sf16, device="b200")
    y = h @ w
    y.status
"""
from __future__ import annotations

from ._array import (DTYPES, SFArray, SFDType, addmm, array, asarray, div, dot, fma, from_codes, full, matmul,
                     resolve_dtype, sqrt, zeros)
from ._array import from_bits
from ._array import sum_ as sum  # noqa: A001
from ._config import accumulate, config, getaccumulate, getconfig, setaccumulate
from ._device import HOST, B200Device, Device, devices, get_device, register_device
from ._errors import *  # noqa: F401,F403
from ._errors import __all__ as _errors_all
from ._errstate import errstate, geterr, seterr
from ._format import FORMATS, MAX_BITS, MIN_BITS, SFFormat
from ._status import SFStatus

__version__ = "0.1.0"

globals().update({f"sf{b}": DTYPES[b] for b in DTYPES})
dtypes = tuple(DTYPES[b] for b in sorted(DTYPES))


def dtype(spec):
    """'sf16', 16 or sf.sf16 -> the sf16 dtype."""
    return resolve_dtype(spec)


def device(name="b200"):
    return get_device(name)


__all__ = ["SFFormat", "FORMATS", "MIN_BITS", "MAX_BITS", "SFStatus", "SFArray", "SFDType", "Device",
           "B200Device", "HOST", "devices", "get_device", "register_device", "device", "errstate", "geterr",
           "seterr", "config", "getconfig", "accumulate", "getaccumulate", "setaccumulate", "array", "asarray",
           "from_codes", "zeros", "full", "matmul", "dot", "addmm", "fma", "div", "sqrt", "sum", "from_bits", "dtype", "dtypes",
           "__version__"] + [f"sf{b}" for b in DTYPES] + list(_errors_all)
