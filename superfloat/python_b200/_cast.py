"""Host-value quantization: float / int / bool arrays -> sfN codes.

The input conversion of ``asarray`` and of literal operands (reference
src/sf/_vectorized.py:32-71): round half to even on the exact scaled value,
saturate where |v| >= 1 - 2^-N (overflow), NaN -> 0 (invalid), a nonzero
value that rounds to 0 (underflow); integers and bools saturate unless 0.
This is input conversion, not the op arithmetic, which runs on the device.
"""
from __future__ import annotations

import numpy as np

from ._format import SFFormat


def cast_array(fmt: SFFormat, values):
    """-> (codes int64, {"overflow", "underflow", "invalid": bool masks})."""
    v = np.asarray(values)
    if v.dtype == object:
        v = v.astype(np.float64)
    if v.dtype.kind in "iub":
        nz = v != 0
        sign = nz.astype(np.int64) if v.dtype.kind in "ub" else np.sign(v).astype(np.int64)
        z = np.zeros(v.shape, bool)
        return sign * fmt.max_code, {"overflow": nz, "underflow": z, "invalid": z.copy()}
    if v.dtype.kind != "f":
        raise TypeError(f"cannot cast array of dtype {v.dtype} to {fmt.name}")
    x = v.astype(np.float64)
    nan = np.isnan(x)
    over = (np.abs(x) >= 1.0 - 2.0 ** -fmt.bits) & ~nan
    ok = ~over & ~nan
    k = np.zeros(x.shape, np.int64)
    k[ok] = np.rint(x[ok] * fmt.scale).astype(np.int64)
    k[over] = np.sign(x[over]).astype(np.int64) * fmt.max_code
    return k, {"overflow": over, "underflow": ok & (k == 0) & (x != 0), "invalid": nan}
