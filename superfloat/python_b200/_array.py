"""SFArray and the array runtime: NumPy-style arrays of one sfN dtype.

Mirrors the reference's array surface (src/sf/_array.py:147-800,
src/sf/_functions.py): ``asarray`` / ``array`` / ``from_codes``, the
arithmetic operators, ``matmul`` / ``dot`` / ``addmm`` with
``accumulate="chain" | "wide"`` and ``shift=``, ``fma`` / ``div`` / ``sqrt``,
``.codes`` / ``.numpy()`` / ``.status``.

Every op's arithmetic runs on a target (the B200 by default) through the
``Device`` interface.  Placement keeps the reference's meaning:

* an op with an operand on a device is *heavy* (src/sf/_array.py:527-591):
  pre-flight gate, launch, exact ``result.status`` from the target's sticky
  per-output events, then the error policy on the status;
* an op on host arrays is *light*: same launch on ``default_device``, and the
  events are raised through the error policy with the reference's messages
  (src/sf/_array.py:34-41); the result stays a host array.
"""
from __future__ import annotations

import numpy as np

from . import _config, _errstate, _preflight
from ._cast import cast_array
from ._device import HOST, get_device
from ._errors import SFShapeError, SFTypeError, SFUnsupportedError
from ._format import FORMATS, SFFormat
from ._status import SFStatus

_SYM = {"add": "+", "sub": "-", "mul": "*", "div": "/", "fma": "fma", "neg": "-", "abs": "abs",
        "sqrt": "sqrt", "pow": "**", "matmul": "@", "matmul_wide": "@ (wide)", "sum": "sum"}
_EVENT_ORDER = ("invalid", "divide", "overflow", "underflow")
_CAN_UNDERFLOW = ("mul", "fma", "matmul", "matmul_wide", "pow")
_COUNT_INDEX = {"overflow": 0, "underflow": 1, "divide": 2, "invalid": 3}


# --- dtypes --------------------------------------------------------------------------------

class SFDType:
    """One sfN dtype (sf4 .. sf16)."""

    __slots__ = ("_fmt", "__name__")

    def __init__(self, bits: int):
        self._fmt = FORMATS[bits]
        self.__name__ = f"sf{bits}"

    @property
    def bits(self) -> int:
        return self._fmt.bits

    def __call__(self, value):
        return SFArray(value, self)

    def __repr__(self):
        return f"sf.{self.__name__}"

    def __reduce__(self):
        return (resolve_dtype, (self._fmt.bits,))


DTYPES = {b: SFDType(b) for b in range(4, 17)}


def resolve_dtype(spec) -> SFDType:
    if isinstance(spec, SFDType):
        return spec
    if isinstance(spec, SFFormat):
        return DTYPES[spec.bits]
    if isinstance(spec, (int, np.integer)) and int(spec) in DTYPES:
        return DTYPES[int(spec)]
    if isinstance(spec, str) and spec.startswith("sf") and spec[2:].isdigit() and int(spec[2:]) in DTYPES:
        return DTYPES[int(spec[2:])]
    raise SFTypeError(f"unknown SF dtype {spec!r}; expected sf4 .. sf16")


# --- operand coercion ------------------------------------------------------------------------

def _handle_events(counts: dict, fmt: SFFormat, opname: str, total: int) -> None:
    for kind in _EVENT_ORDER:
        n = counts.get(kind, 0)
        if n:
            _errstate.handle(kind, f"{fmt.name} {opname}: {kind} in {n} of {total} element(s)")


def _widest(xs) -> SFFormat:
    fmts = [x.dtype._fmt for x in xs if isinstance(x, SFArray)]
    if not fmts:
        raise SFTypeError("at least one operand must be an SF array")
    return max(fmts, key=lambda f: f.bits)


def _device_of(xs) -> str:
    devs = {x.device for x in xs if isinstance(x, SFArray) and x.device != HOST}
    if len(devs) > 1:
        raise SFTypeError(f"operands live on different devices: {sorted(devs)}")
    return devs.pop() if devs else HOST


def _to_codes(x, fmt: SFFormat, what: str = "literal") -> np.ndarray:
    """Any operand -> int64 codes in ``fmt``: SF arrays are widened (never
    narrowed), host numbers are quantized through the error policy."""
    if isinstance(x, SFArray):
        if x.dtype._fmt.bits > fmt.bits:
            raise SFTypeError(f"cannot store {x.dtype.__name__} into {fmt.name} implicitly; use sf.cast")
        return x._codes << (fmt.bits - x.dtype._fmt.bits)
    if isinstance(x, (str, bytes)):
        raise SFTypeError(f"cannot use {type(x).__name__} as an SF operand")
    arr = np.asarray(x)
    if arr.dtype.kind not in "fiubO":
        raise SFTypeError(f"cannot use {arr.dtype} data as an SF operand")
    try:
        codes, ev = cast_array(fmt, arr)
    except (TypeError, ValueError) as e:
        raise SFTypeError(str(e)) from None
    _handle_events({k: int(np.count_nonzero(m)) for k, m in ev.items()}, fmt, f"{what} cast", max(1, arr.size))
    return codes


# --- the array type --------------------------------------------------------------------------

class SFArray:
    """N-dimensional array of one SF dtype: int64 codes on the host, placed on
    ``device`` for heavy ops."""

    __slots__ = ("_codes", "_dtype", "_device", "_status", "_events")
    __array_ufunc__ = None

    def __init__(self, obj, dtype=None, device: str = HOST):
        if isinstance(obj, SFArray) and dtype is None:
            dtype = obj.dtype
        if dtype is None:
            raise SFTypeError("sf.array needs dtype= unless the input already holds SF values")
        cls = resolve_dtype(dtype)
        self._codes = np.array(_to_codes(obj, cls._fmt, what="value"), dtype=np.int64, copy=True)
        self._dtype = cls
        self._device = HOST
        self._status = None
        self._events = None
        if device != HOST:
            d = get_device(device)
            d.check(cls._fmt, self._codes.size)
            self._device = d.name

    @classmethod
    def _wrap(cls, codes, dtype, device: str = HOST, status=None):
        obj = object.__new__(cls)
        obj._codes = np.asarray(codes, dtype=np.int64)
        obj._dtype = dtype
        obj._device = device
        obj._status = status
        obj._events = None
        return obj

    dtype = property(lambda self: self._dtype)
    device = property(lambda self: self._device)
    status = property(lambda self: self._status, doc="Status of the heavy op that produced this array.")
    shape = property(lambda self: self._codes.shape)
    ndim = property(lambda self: self._codes.ndim)
    size = property(lambda self: self._codes.size)

    @property
    def codes(self) -> np.ndarray:
        v = self._codes.view()
        v.flags.writeable = False
        return v

    @property
    def bits(self) -> np.ndarray:
        """Sign-magnitude device patterns (uint16), as src/sf/_vectorized.py:78-82."""
        fmt = self._dtype._fmt
        k = self._codes
        return np.where(k < 0, (1 << fmt.frac_bits) | (-k), k).astype(np.uint16)

    def numpy(self) -> np.ndarray:
        return self._codes.astype(np.float64) / self._dtype._fmt.scale

    def tolist(self):
        return self.numpy().tolist()

    def to(self, device: str) -> "SFArray":
        if device == HOST:
            return SFArray._wrap(self._codes.copy(), self._dtype)
        d = get_device(device)
        d.check(self._dtype._fmt, self.size)
        return SFArray._wrap(self._codes.copy(), self._dtype, d.name)

    def copy(self):
        return SFArray._wrap(self._codes.copy(), self._dtype, self._device, self._status)

    def reshape(self, *shape):
        if len(shape) == 1 and isinstance(shape[0], (tuple, list)):
            shape = tuple(shape[0])
        return SFArray._wrap(self._codes.reshape(shape), self._dtype, self._device)

    @property
    def T(self):
        return SFArray._wrap(self._codes.T, self._dtype, self._device)

    def transpose(self, *axes):
        return SFArray._wrap(self._codes.transpose(*axes) if axes else self._codes.T, self._dtype, self._device)

    def flatten(self):
        return SFArray._wrap(self._codes.flatten(), self._dtype, self._device)

    def __len__(self):
        if self.ndim == 0:
            raise TypeError("len() of a 0-d SF array")
        return self._codes.shape[0]

    def __getitem__(self, idx):
        if isinstance(idx, SFArray):
            raise SFTypeError("SF arrays cannot be used as indices")
        return SFArray._wrap(np.asarray(self._codes[idx]), self._dtype, self._device)

    def __setitem__(self, idx, value):
        self._codes[idx] = _to_codes(value, self._dtype._fmt, what="value")

    def __repr__(self):
        body = np.array2string(self.numpy(), separator=", ", threshold=50)
        extra = f", device='{self._device}'" if self._device != HOST else ""
        return f"sfarray({body}, dtype={self._dtype.__name__}{extra})"

    __str__ = __repr__

    def __float__(self):
        if self.size != 1:
            raise TypeError("only size-1 SF arrays can be converted to float")
        return float(self.numpy().reshape(()))

    def any(self):
        return bool(np.any(self._codes))

    def all(self):
        return bool(np.all(self._codes))

    def __bool__(self):
        if self.size != 1:
            raise ValueError("the truth value of an SF array with more than one element is ambiguous")
        return bool(self._codes.reshape(()) != 0)

    def __eq__(self, o):
        return self.numpy() == (o.numpy() if isinstance(o, SFArray) else np.asarray(o, dtype=np.float64))

    def __ne__(self, o):
        return ~self.__eq__(o)

    __hash__ = None

    # operators (src/sf/_array.py:318-349)
    def __add__(self, o): return _elementwise("add", self, o)
    def __radd__(self, o): return _elementwise("add", o, self)
    def __sub__(self, o): return _elementwise("sub", self, o)
    def __rsub__(self, o): return _elementwise("sub", o, self)
    def __mul__(self, o): return _elementwise("mul", self, o)
    def __rmul__(self, o): return _elementwise("mul", o, self)
    def __truediv__(self, o): return _elementwise("div", self, o)
    def __rtruediv__(self, o): return _elementwise("div", o, self)
    def __neg__(self): return _elementwise("neg", self)
    def __pos__(self): return self
    def __abs__(self): return _elementwise("abs", self)
    def sum(self, axis=None):
        return sum_(self, axis)

    def __matmul__(self, o): return matmul(self, o)
    def __rmatmul__(self, o): return matmul(o, self)

    def __pow__(self, n, mod=None):
        if mod is not None or isinstance(n, bool) or not isinstance(n, (int, np.integer)):
            raise SFUnsupportedError("only integer exponents k >= 1 are supported")
        n = int(n)
        if n == 0:
            fmt = self._dtype._fmt
            _errstate.handle("overflow", f"x ** 0 = 1 is not representable in {fmt.name}")
            return SFArray._wrap(np.full(self.shape, fmt.max_code, np.int64), self._dtype, self._device)
        if n < 0:
            raise SFUnsupportedError("negative exponents overflow for every nonzero SF value")
        return _elementwise("pow", self, n=n)

    def __reduce__(self):
        return (_rebuild, (self._codes, self._dtype._fmt.bits, self._device))


def _rebuild(codes, bits, device):
    return SFArray._wrap(codes, DTYPES[bits], device)


# --- constructors ----------------------------------------------------------------------------

def array(obj, dtype=None, device: str = HOST) -> SFArray:
    return SFArray(obj, dtype, device)


def asarray(obj, dtype=None, device: str = HOST) -> SFArray:
    if isinstance(obj, SFArray) and (dtype is None or resolve_dtype(dtype) is obj.dtype) and obj.device == device:
        return obj
    return SFArray(obj, dtype, device)


def from_codes(codes, dt, device: str = HOST) -> SFArray:
    cls = resolve_dtype(dt)
    k = np.asarray(codes)
    if k.dtype.kind not in "iu":
        raise SFTypeError("codes must be an integer array")
    if k.size and (int(k.max()) > cls._fmt.max_code or int(k.min()) < -cls._fmt.max_code):
        from ._errors import SFInvalidError
        raise SFInvalidError(f"codes outside {cls.__name__} range ±{cls._fmt.max_code}")
    out = SFArray._wrap(k.astype(np.int64), cls)
    return out if device == HOST else out.to(device)


def from_bits(bits, dt, device: str = HOST) -> SFArray:
    """Sign-magnitude words (the chip's memory format) -> an SF array: sign at
    bit N-1, |k| in the low N-1 bits, the sign-only word reads as 0;
    ValueError for a word that does not fit (src/sf/_vectorized.py:84-89,
    src/sf/_functions.py:136-144)."""
    dt = resolve_dtype(dt)
    fmt = FORMATS[dt.bits]
    b = np.asarray(bits)
    if b.dtype == bool or not np.issubdtype(b.dtype, np.integer):
        raise TypeError(f"bits must be integers, got {b.dtype}")
    b = b.astype(np.int64)
    if np.any((b < 0) | (b >= (1 << fmt.bits))):
        raise ValueError(f"bit pattern does not fit in {fmt.bits} bits")
    mag = b & fmt.max_code
    return SFArray._wrap(np.where(b >> fmt.frac_bits, -mag, mag).astype(np.int64), dt, device)


def zeros(shape, dtype="sf16", device: str = HOST) -> SFArray:
    out = SFArray._wrap(np.zeros(shape, np.int64), resolve_dtype(dtype))
    return out if device == HOST else out.to(device)


def full(shape, value, dtype, device: str = HOST) -> SFArray:
    cls = resolve_dtype(dtype)
    k = int(_to_codes(value, cls._fmt, what="value"))
    out = SFArray._wrap(np.full(shape, k, np.int64), cls)
    return out if device == HOST else out.to(device)


# --- the engine --------------------------------------------------------------------------------

def _launch(dev, op, fmt, codes, out_shape, kw):
    """Run on the target: int64 codes in, (int64 codes of out_shape, event counts) out."""
    if hasattr(dev, "launches"):
        dev.launches += 1
    if not hasattr(dev, "run_device"):                     # a plain Device: the masks contract
        res, flags = dev.run(op, fmt, *codes, **kw)
        res = np.broadcast_to(np.asarray(res, np.int64), out_shape).copy()
        return res, {k: int(np.count_nonzero(v)) for k, v in (flags or {}).items()}
    if int(np.prod(out_shape)) == 0:
        return np.zeros(out_shape, np.int64), {}
    ts = [dev.upload(c) for c in codes]
    out, cnt, _ = dev.run_device(op, fmt, *ts, **kw)
    res = out.cpu().numpy().astype(np.int64)
    c = cnt.cpu().numpy()
    from . import _lib
    _lib.check_counts(c)
    res = np.broadcast_to(res, out_shape).copy() if res.shape != tuple(out_shape) else res
    return res, {k: int(c[i]) for k, i in _COUNT_INDEX.items()}


def _elementwise(op, *xs, **kw):
    fmt = _widest(xs)
    dtype = DTYPES[fmt.bits]
    device = _device_of(xs)
    codes = [_to_codes(x, fmt) for x in xs]
    try:
        shape = np.broadcast_shapes(*(c.shape for c in codes))
    except ValueError:
        raise SFShapeError(f"operands could not be broadcast together: {[c.shape for c in codes]}") from None
    total = int(np.prod(shape)) if shape else 1
    if device == HOST and not _should_offload(total, op, fmt):
        dev = get_device(_config.get("default_device"))
        res, counts = _launch(dev, op, fmt, codes, shape, kw)
        _handle_events(counts, fmt, _SYM[op], total)
        return SFArray._wrap(res, dtype)
    target = device if device != HOST else _config.get("default_device")
    return _run_heavy(op, fmt, dtype, target, codes, shape, kw)


def _should_offload(total, op, fmt) -> bool:
    t = _config.get("offload_threshold")
    if t is None or total <= t:
        return False
    dev = get_device(_config.get("default_device"))
    if dev.supported_ops is not None and op not in dev.supported_ops:
        return False
    if op == "matmul_wide" and not dev.mx:
        return False
    return fmt.bits in dev.widths_for(op)


def _run_heavy(op, fmt, dtype, device, codes, out_shape, kw):
    """Pre-flight, launch, status (src/sf/_array.py:527-591)."""
    dev = get_device(device)
    if op == "matmul_wide" and dev.mx:
        kw = {**kw, "mx": dev.mx}
    dev.check(fmt, max(int(np.prod(out_shape)) if out_shape else 1, *(c.size for c in codes)), op)
    opname = _SYM[op]
    verdict = _preflight.check(op, fmt, *codes, **kw)
    if verdict.events.get("invalid"):
        _errstate.handle("invalid", f"{fmt.name} {opname} on {dev.name}: invalid in "
                                    f"{verdict.events['invalid']} element(s) (status.invalid)")
    if verdict.events.get("div0"):
        _errstate.handle("divide", f"{fmt.name} {opname} on {dev.name}: division by zero in "
                                   f"{verdict.events['div0']} element(s) (status.div0)")
    verdict = _preflight.decide(verdict, op, fmt, dev, *codes, **kw)
    if dev.supported_ops is not None and op not in dev.supported_ops:
        raise SFUnsupportedError(f"{fmt.name} {opname} has no instruction on {dev.name}; nothing was launched")
    res, counts = _launch(dev, op, fmt, codes, out_shape, kw)
    at_max = int(np.count_nonzero(np.abs(res) == fmt.max_code))
    status = SFStatus(saturated=counts.get("overflow", 0), div0=verdict.events.get("div0", 0),
                      invalid=verdict.events.get("invalid", 0), exact=True, outputs_at_max=at_max,
                      underflow=counts.get("underflow", 0) if op in _CAN_UNDERFLOW else 0)
    if status.saturated:
        _errstate.handle("overflow", f"{fmt.name} {opname} on {dev.name}: saturation in "
                                     f"{status.saturated} element(s) (status.saturated)")
    if status.underflow:
        _errstate.handle("underflow", f"{fmt.name} {opname} on {dev.name}: underflow in "
                                      f"{status.underflow} element(s) (status.underflow)")
    return SFArray._wrap(res, dtype, dev.name, status)


# --- linear algebra ------------------------------------------------------------------------------

def _as_sfarray(x, name) -> SFArray:
    if isinstance(x, SFArray):
        return x
    raise SFTypeError(f"sf.{name} expects SF arrays (got {type(x).__name__}); convert host data with "
                      "sf.asarray(x, dtype=...)")


def _mode_and_shift(accumulate, shift, name):
    from ._config import resolve_mode
    mode = resolve_mode(accumulate)
    if mode == "chain":
        if shift is not None:
            raise ValueError(f"sf.{name}: shift= only applies to accumulate=\"wide\" (this call accumulates "
                             f"as 'chain')")
        return mode, 0
    return mode, _check_shift(shift, name)


def _check_shift(shift, name):
    """An int in -32..31 or an integer array of them (src/sf/_linalg.py:223-247)."""
    if shift is None:
        return 0
    if isinstance(shift, (bool, np.bool_)):
        raise TypeError(f"sf.{name}: shift must be an int or an array of ints, got bool")
    if isinstance(shift, (int, np.integer)):
        if not -32 <= int(shift) <= 31:
            raise ValueError(f"sf.{name}: shift must be between -32 and 31, got {shift}")
        return int(shift)
    arr = np.asarray(shift)
    if arr.dtype == bool or not np.issubdtype(arr.dtype, np.integer):
        raise TypeError(f"sf.{name}: shift must be an int or an array of ints, got an array of {arr.dtype}")
    if arr.size and (arr.min() < -32 or arr.max() > 31):
        raise ValueError(f"sf.{name}: every shift must be between -32 and 31")
    arr = arr.astype(np.int64)
    return int(arr) if arr.ndim == 0 else arr


def matmul(a, b, *, accumulate=None, shift=None):
    """``a @ b`` with NumPy's rules for 1-D operands and batching
    (src/sf/_array.py:730-792).  ``accumulate="chain"`` (default) or
    ``"wide"`` with ``shift`` an int or an int array broadcastable to the
    result."""
    mode, sh = _mode_and_shift(accumulate, shift, "matmul")
    a, b = _as_sfarray(a, "matmul"), _as_sfarray(b, "matmul")
    if a.ndim == 0 or b.ndim == 0:
        raise SFShapeError("matmul: operands must be at least 1-D (use * for scalars)")
    fmt = _widest([a, b])
    dtype = DTYPES[fmt.bits]
    ka, kb = _to_codes(a, fmt), _to_codes(b, fmt)
    sq_row = sq_col = False
    if ka.ndim == 1:
        ka, sq_row = ka[None, :], True
    if kb.ndim == 1:
        kb, sq_col = kb[:, None], True
    if ka.shape[-1] != kb.shape[-2]:
        raise SFShapeError(f"matmul: shapes {a.shape} and {b.shape} are not aligned "
                           f"({ka.shape[-1]} != {kb.shape[-2]})")
    try:
        batch = np.broadcast_shapes(ka.shape[:-2], kb.shape[:-2])
    except ValueError:
        raise SFShapeError(f"matmul: batch shapes {ka.shape[:-2]} and {kb.shape[:-2]} cannot be broadcast") \
            from None
    out_shape = batch + (ka.shape[-2], kb.shape[-1])
    if not isinstance(sh, int):
        seen = out_shape[:-2] + (() if sq_row else out_shape[-2:-1]) + (() if sq_col else out_shape[-1:])
        try:
            sh = np.ascontiguousarray(np.broadcast_to(sh, seen)).reshape(out_shape)
        except ValueError:
            raise SFShapeError(f"sf.matmul: shift of shape {sh.shape} does not broadcast to the result shape "
                               f"{tuple(seen)}") from None
    op, kw = ("matmul_wide", {"shift": sh}) if mode == "wide" else ("matmul", {})
    device = _device_of([a, b])
    total = int(np.prod(out_shape))
    if device == HOST and not _should_offload(total * ka.shape[-1], op, fmt):
        dev = get_device(_config.get("default_device"))
        if op == "matmul_wide":
            kw = {**kw, "mx": dev.mx or "v4.9.2"}
        res, counts = _launch(dev, op, fmt, [ka, kb], out_shape, kw)
        _handle_events(counts, fmt, _SYM[op], total)
        out = SFArray._wrap(res, dtype)
    else:
        target = device if device != HOST else _config.get("default_device")
        out = _run_heavy(op, fmt, dtype, target, [ka, kb], out_shape, kw)
    codes = out._codes
    if sq_row:
        codes = codes[..., 0, :]
    if sq_col:
        codes = codes[..., 0]
    return SFArray._wrap(codes, dtype, out.device, out.status)


def dot(a, b, *, accumulate=None, shift=None):
    """1-D . 1-D (chain of fma, or the MX engine); higher ranks go to matmul."""
    a, b = _as_sfarray(a, "dot"), _as_sfarray(b, "dot")
    if a.ndim == 1 and b.ndim == 1 and a.shape != b.shape:
        raise SFShapeError(f"sf.dot: shapes {a.shape} and {b.shape} differ")
    return matmul(a, b, accumulate=accumulate, shift=shift)


def sum_(x, axis=None):
    """Saturating sum along ``axis`` (every element when None), index 0 first:
    the reference's sequential order (src/sf/_array.py:636-656)."""
    x = _as_sfarray(x, "sum")
    fmt = FORMATS[x.dtype.bits]
    codes = x.codes
    if axis is None:
        codes, axis = codes.reshape(-1), 0
    elif axis < 0:
        axis += codes.ndim
    if not 0 <= axis < codes.ndim:
        raise SFShapeError(f"axis {axis} is out of bounds for an array of dimension {codes.ndim}")
    out_shape = codes.shape[:axis] + codes.shape[axis + 1:]
    kw = {"axis": axis}
    if x.device == HOST and not _should_offload(codes.size, "sum", fmt):
        dev = get_device(_config.get("default_device"))
        res, counts = _launch(dev, "sum", fmt, [codes], out_shape, kw)
        _handle_events(counts, fmt, "sum", int(np.prod(out_shape)) if out_shape else 1)
        return SFArray._wrap(res, x.dtype)
    target = x.device if x.device != HOST else _config.get("default_device")
    return _run_heavy("sum", fmt, x.dtype, target, [codes], out_shape, kw)


def addmm(a, b, d, *, accumulate=None, shift=None):
    """``a @ b + d``: the matmul, then one saturating add of ``d``."""
    return matmul(a, b, accumulate=accumulate, shift=shift) + d


def fma(a, b, c):
    """a * b + c with the reference's two roundings (bit-identical to a * b + c)."""
    return _elementwise("fma", a, b, c)


def div(a, b, where=None):
    """a / b; with ``where=mask`` only where the mask is True (0 elsewhere, no events)."""
    if where is None:
        return _elementwise("div", a, b)
    fmt = _widest([a, b])
    ka, kb = _to_codes(a, fmt), _to_codes(b, fmt)
    mask = np.asarray(where, dtype=bool)
    try:
        shape = np.broadcast_shapes(ka.shape, kb.shape, mask.shape)
    except ValueError:
        raise SFShapeError("sf.div: operands and mask could not be broadcast together") from None
    ka, kb, mask = (np.broadcast_to(v, shape) for v in (ka, kb, mask))
    dev_name = _device_of([a, b])
    sub_a = SFArray._wrap(ka[mask], DTYPES[fmt.bits], dev_name)
    sub_b = SFArray._wrap(kb[mask], DTYPES[fmt.bits], dev_name)
    part = _elementwise("div", sub_a, sub_b)
    res = np.zeros(shape, np.int64)
    res[mask] = part._codes
    return SFArray._wrap(res, DTYPES[fmt.bits], part.device, part.status)


def sqrt(a):
    """Square root truncated toward zero; a negative input is invalid (device value 0)."""
    return _elementwise("sqrt", _as_sfarray(a, "sqrt"))
