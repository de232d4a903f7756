"""Targets: the ``Device`` plug-in interface and the B200 target.

``Device`` mirrors the reference's target interface (src/sf/_device.py:38-106):
attributes ``name``, ``supported_bits``, ``accumulation_order``,
``accumulator_bits``, ``sticky_flags``, ``max_elements``, ``supported_ops``,
``mx``, ``wide_bits``; methods ``widths_for``, ``can_run``, ``check`` and
``run(op, fmt, *codes, **kw) -> (codes, flags)``.

``B200Device`` is the drop-in: ``run`` takes the reference's operands (int64
NumPy code arrays, broadcastable, caller-owned) and returns int64 codes of the
output shape plus per-output boolean event masks, with the sticky-flags
contract of the reference's flagged target (src/sf/_device.py:151-163).  The
work runs in libsfb200 on an sm_100 GPU; there is no CPU fallback.  The
same object also runs on device-resident torch int16 code tensors
(``run_device``), which is what this package's array runtime and torch layers
use.  A maintainer adds it to the reference's own runtime with
``sf.register_device(B200Device())`` (it is duck-compatible with sf.Device).
"""
from __future__ import annotations

import threading
import warnings

import numpy as np

from . import _lib
from ._errors import SFLaunchError, SFShapeError, SFUnsupportedError
from ._format import SFFormat

HOST = "host"

# the events each op can raise: the keys of the masks ``run`` returns, as the
# reference's flagged target returns them (src/sf/_vectorized.py:94-156,
# src/sf/_linalg.py:61-81, :330-348)
OP_EVENTS = {
    "add": ("overflow",), "sub": ("overflow",), "mul": ("underflow",), "div": ("overflow", "divide"),
    "fma": ("overflow", "underflow"), "neg": (), "abs": (), "sqrt": ("invalid",), "pow": ("underflow",),
    "matmul": ("overflow", "underflow"), "matmul_wide": ("overflow", "underflow"), "sum": ("overflow",),
}
_EVENT_BIT = {"overflow": _lib.F_OVERFLOW, "underflow": _lib.F_UNDERFLOW, "divide": _lib.F_DIVIDE,
              "invalid": _lib.F_INVALID}
# elementwise Device.run calls at least this large (all operands of the
# output's shape) go through the pooled, chunked host pipeline
STAGED_MIN_ELEMENTS = 1 << 20

ARITY = {"add": 2, "sub": 2, "mul": 2, "div": 2, "fma": 3, "neg": 1, "abs": 1, "sqrt": 1, "pow": 1,
         "matmul": 2, "matmul_wide": 2, "sum": 1}


class Device:
    """Base class of every target (src/sf/_device.py:38-106)."""

    name: str = ""
    supported_bits: tuple = ()
    accumulation_order: str = "sequential"
    accumulator_bits = None
    sticky_flags: bool = False
    max_elements = None
    supported_ops = None
    mx = False
    wide_bits: tuple = ()

    def widths_for(self, op=None) -> tuple:
        wide = (self.wide_bits or self.supported_bits) if self.mx else ()
        if op == "matmul_wide":
            return wide
        if op is None:
            return tuple(sorted(set(self.supported_bits) | set(wide)))
        return self.supported_bits

    def can_run(self, op, fmt) -> bool:
        if self.supported_ops is not None and op not in self.supported_ops:
            return False
        return fmt.bits in self.widths_for(op)

    def check(self, fmt: SFFormat, n_elements: int, op=None) -> None:
        if op == "matmul_wide" and not self.mx:
            raise SFUnsupportedError(f"{self.name} has no MX engine, so accumulate=\"wide\" cannot run "
                                     f"there; nothing was launched")
        if fmt.bits not in self.widths_for(op):
            raise SFUnsupportedError(f"{fmt.name} is not supported on {self.name}")
        if self.max_elements is not None and n_elements > self.max_elements:
            raise SFLaunchError(f"{n_elements} elements exceed the {self.name} limit of {self.max_elements}")

    def run(self, op, fmt, *operands, **kw):
        raise NotImplementedError

    def __repr__(self):
        return f"<sf device {self.name}>"


def _torch():
    import torch
    return torch


class B200Device(Device):
    """An sm_100 GPU running libsfb200's kernels (the drop-in target)."""

    name = "b200"
    supported_bits = tuple(range(4, 17))
    wide_bits = tuple(range(4, 17))
    accumulation_order = "sequential"
    accumulator_bits = None
    sticky_flags = True
    max_elements = 1 << 34
    mx = "v4.9.2"
    supported_ops = frozenset({"add", "sub", "mul", "div", "fma", "neg", "abs", "sqrt", "pow",
                               "matmul", "matmul_wide", "sum"})

    def __init__(self, index: int = 0, *, mx=None, name=None):
        if mx is not None:
            if mx not in _lib.MX:
                raise ValueError(f"unknown MX version {mx!r}; expected one of {tuple(_lib.MX)}")
            self.mx = mx
        if name is not None:
            self.name = name
        self.index = index
        self.launches = 0
        self._lock = threading.Lock()
        self._ws = None
        self._stager = None

    # --- device plumbing -------------------------------------------------------------------
    @property
    def torch_device(self):
        return _torch().device("cuda", self.index)

    def _ready(self):
        torch = _torch()
        if not torch.cuda.is_available():
            from ._errors import SFDeviceError
            raise SFDeviceError("the b200 target needs a CUDA device; none is visible")
        _lib.ensure_device(self.index)
        return torch

    def counts_buffer(self):
        torch = self._ready()
        return torch.zeros(_lib.N_COUNTS, dtype=torch.int64, device=self.torch_device)

    def workspace(self, nbytes: int):
        """A cached device workspace of at least ``nbytes`` (grown, never shrunk)."""
        torch = self._ready()
        if nbytes <= 0:
            return None
        if self._ws is None or self._ws.numel() < nbytes:
            self._ws = torch.empty(nbytes, dtype=torch.uint8, device=self.torch_device)
        return self._ws

    def upload(self, codes: np.ndarray):
        """int64 host codes -> int16 device tensor (same shape)."""
        torch = self._ready()
        with warnings.catch_warnings():
            warnings.simplefilter("ignore")          # a read-only caller array: it is only read here
            host = torch.from_numpy(np.ascontiguousarray(codes)).to(torch.int16)
        return host.pin_memory().to(self.torch_device, non_blocking=True)

    # --- device-resident execution ---------------------------------------------------------
    def run_device(self, op, fmt, *xs, flags=False, counts=None, out=None, stream=None, **kw):
        """Run ``op`` on int16 code tensors on this device.  Returns
        (codes tensor, counts tensor int64[8], flags tensor uint8 or None).
        ``counts`` accumulates when given (zeroed by the caller)."""
        torch = self._ready()
        dev = self.torch_device
        cnt = counts if counts is not None else torch.zeros(_lib.N_COUNTS, dtype=torch.int64, device=dev)
        bits = fmt.bits
        if op in ("matmul", "matmul_wide"):
            return self._matmul_device(op, fmt, xs[0], xs[1], flags, cnt, out, stream, **kw)
        if op == "sum":
            return self._sum_device(fmt, xs[0], _axis(kw.get("axis", 0), xs[0].dim()), flags, cnt, out, stream)
        shape = torch.broadcast_shapes(*(x.shape for x in xs))
        xs = [x if (tuple(x.shape) == tuple(shape) and x.is_contiguous()) else x.expand(shape).contiguous()
              for x in xs]
        o = out if out is not None else torch.empty(shape, dtype=torch.int16, device=dev)
        fl = torch.empty(shape, dtype=torch.uint8, device=dev) if flags else None
        a = xs[0]
        b = xs[1] if len(xs) > 1 else None
        c = xs[2] if len(xs) > 2 else None
        _lib.elementwise(op, bits, a, b, c, o, fl, cnt, pow_n=int(kw.get("n", 0)), stream=stream)
        return o, cnt, fl

    def _matmul_device(self, op, fmt, A, B, flags, cnt, out, stream, shift=0, mx=None, bias=None):
        torch = _torch()
        if A.dim() < 2 or B.dim() < 2:
            raise SFShapeError("matmul operands must be at least 2-D here")
        M, K = A.shape[-2], A.shape[-1]
        K2, N = B.shape[-2], B.shape[-1]
        if K != K2:
            raise SFShapeError(f"matmul: shapes {tuple(A.shape)} and {tuple(B.shape)} are not aligned")
        batch_shape = torch.broadcast_shapes(A.shape[:-2], B.shape[:-2])
        nb = int(np.prod(batch_shape)) if len(batch_shape) else 1
        A3, sa = _batched(A, batch_shape, nb)
        B3, sb = _batched(B, batch_shape, nb)
        o = out if out is not None else torch.empty(tuple(batch_shape) + (M, N), dtype=torch.int16,
                                                    device=A.device)
        fl = torch.empty(tuple(batch_shape) + (M, N), dtype=torch.uint8, device=A.device) if flags else None
        if op == "matmul" and nb == 1 and M == 1 and N == 1 and bias is None and K > 0:
            # one chain: the ordered parallel reduction (same bits as the chain kernel)
            a1, b1 = A3.reshape(K).contiguous(), B3.reshape(K).contiguous()
            ws = self.workspace(_lib.reduce_workspace(1, K))
            _lib.dot(fmt.bits, a1, b1, K, o, fl, ws, cnt, stream=stream)
        elif op == "matmul":
            ws = self.workspace(_lib.chain_workspace(nb, M, N, K))
            _lib.matmul_chain_ws(fmt.bits, A3, B3, bias, o, fl, cnt, nb, M, N, K, _ld(A3), _ld(B3),
                                 sa, sb, M * N, ws, stream=stream)
        else:
            mxv = mx or self.mx
            sh_t = None
            sh_int = 0
            ss = (0, 0, 0)
            if isinstance(shift, (int, np.integer)):
                sh_int = int(shift)
            else:
                st = shift if hasattr(shift, "data_ptr") else torch.as_tensor(np.asarray(shift), device=A.device)
                st = st.to(device=A.device, dtype=torch.int8).expand(tuple(batch_shape) + (M, N))
                st = st.reshape(nb, M, N) if nb > 1 or len(batch_shape) else st.reshape(1, M, N)
                sh_t = st
                ss = (st.stride(0), st.stride(1), st.stride(2))
            ws = self.workspace(_lib.wide_workspace(fmt.bits, mxv, nb, M, N, K))
            _lib.matmul_wide(fmt.bits, mxv, A3, B3, sh_t, sh_int, o, fl, cnt, nb, M, N, K, _ld(A3), _ld(B3),
                             sa, sb, M * N, ss[0], ss[1], ss[2], ws, stream=stream)
        return o, cnt, fl

    def _sum_device(self, fmt, X, axis, flags, cnt, out, stream):
        """Saturating sequential sum of int16 codes along ``axis``."""
        torch = _torch()
        X = X.contiguous()
        shape = tuple(X.shape)
        K = shape[axis]
        outer = int(np.prod(shape[:axis])) if axis else 1
        inner = int(np.prod(shape[axis + 1:])) if axis + 1 < len(shape) else 1
        oshape = shape[:axis] + shape[axis + 1:]
        o = out if out is not None else torch.empty(oshape, dtype=torch.int16, device=X.device)
        fl = torch.empty(oshape, dtype=torch.uint8, device=X.device) if flags else None
        ws = self.workspace(_lib.reduce_workspace(outer, K) if inner == 1 else 0)
        _lib.sum_codes(fmt.bits, X, outer, K, inner, o, fl, ws, cnt, stream=stream)
        return o, cnt, fl

    # --- the chip's sign-magnitude memory format -------------------------------------------
    def upload_bits(self, fmt, patterns):
        """Sign-magnitude words (host) -> int16 device codes, converted on the
        device; ValueError for a word that does not fit ``fmt``'s width
        (src/sf/_vectorized.py:84-89)."""
        torch = self._ready()
        p = np.asarray(patterns)
        if p.size and (p.min() < 0 or p.max() >= (1 << 16)):
            raise ValueError(f"bit pattern does not fit in {fmt.bits} bits")
        host = torch.from_numpy(np.ascontiguousarray(p, dtype=np.uint16).view(np.int16))
        words = host.pin_memory().to(self.torch_device, non_blocking=True)
        codes = torch.empty_like(words)
        cnt = torch.zeros(_lib.N_COUNTS, dtype=torch.int64, device=self.torch_device)
        _lib.from_bits(fmt.bits, words, codes, cnt)
        _lib.check_patterns(cnt.cpu().numpy(), fmt.bits)
        return codes

    def download_bits(self, fmt, codes) -> np.ndarray:
        """int16 device codes -> sign-magnitude words (host uint16)."""
        torch = self._ready()
        words = torch.empty_like(codes)
        _lib.to_bits(fmt.bits, codes.contiguous(), words)
        return words.cpu().numpy().view(np.uint16)

    def run_bits(self, op, fmt, *patterns, **kw):
        """``run`` in the chip's format: sign-magnitude words in and out.
        Elementwise ops read and write the words directly in the kernel;
        reductions convert on the device around the code kernels.  Returns
        (uint16 words, event masks)."""
        torch = self._ready()
        with self._lock:
            self.launches += 1
        if op in ("matmul", "matmul_wide", "sum"):
            xs = [self.upload_bits(fmt, p) for p in patterns[:ARITY[op]]]
            codes, cnt, fl = self.run_device(op, fmt, *xs, flags=True, **kw)
            _lib.check_counts(cnt.cpu().numpy())
            words = self.download_bits(fmt, codes)
        else:
            ps = [np.asarray(p) for p in patterns[:ARITY[op]]]
            for p in ps:
                if p.size and (p.min() < 0 or p.max() >= (1 << 16)):
                    raise ValueError(f"bit pattern does not fit in {fmt.bits} bits")
            shape = np.broadcast_shapes(*(p.shape for p in ps))
            xs = [torch.from_numpy(np.array(np.broadcast_to(p, shape), dtype=np.uint16).view(np.int16))
                  .to(self.torch_device) for p in ps]
            out = torch.empty(shape, dtype=torch.int16, device=self.torch_device)
            fl = torch.empty(shape, dtype=torch.uint8, device=self.torch_device)
            cnt = torch.zeros(_lib.N_COUNTS, dtype=torch.int64, device=self.torch_device)
            if out.numel():
                _lib.elementwise_signmag(op, fmt.bits, xs[0], xs[1] if len(xs) > 1 else None,
                                         xs[2] if len(xs) > 2 else None, out, fl, cnt, pow_n=int(kw.get("n", 0)))
            c = cnt.cpu().numpy()
            _lib.check_counts(c)
            _lib.check_patterns(c, fmt.bits)
            words = out.cpu().numpy().view(np.uint16)
        fl = fl.cpu().numpy()
        return words, {e: (fl & _EVENT_BIT[e]) != 0 for e in OP_EVENTS[op]}

    # --- the reference's plug-in contract --------------------------------------------------
    def run(self, op, fmt, *operands, **kw):
        """Execute ``op`` on int64 code arrays (src/sf/_device.py:96-106).
        Returns ``(codes, flags)``: int64 codes of the broadcast output shape
        and a dict of boolean masks for the events ``op`` can raise.  Counts
        one launch in ``launches``."""
        with self._lock:
            self.launches += 1
        return self.evaluate(op, fmt, *operands, **kw)

    def evaluate(self, op, fmt, *operands, **kw):
        """``run`` without counting a launch: the pre-flight probe and replay
        use it, so ``launches`` counts only the ops the runtime committed to."""
        if op not in ARITY:
            raise SFUnsupportedError(f"{op} is not an op of the {self.name} target")
        ops = [np.asarray(o, dtype=np.int64) for o in operands[:ARITY[op]]]
        if op in ("matmul", "matmul_wide"):
            out_shape = np.broadcast_shapes(ops[0].shape[:-2], ops[1].shape[:-2]) + (ops[0].shape[-2],
                                                                                       ops[1].shape[-1])
        elif op == "sum":
            axis = _axis(kw.get("axis", 0), ops[0].ndim)
            kw = {"axis": axis}
            out_shape = ops[0].shape[:axis] + ops[0].shape[axis + 1:]
        else:
            out_shape = np.broadcast_shapes(*(o.shape for o in ops))
        if int(np.prod(out_shape)) == 0:
            return np.zeros(out_shape, np.int64), {e: np.zeros(out_shape, bool) for e in OP_EVENTS[op]}
        if (op not in ("matmul", "matmul_wide", "sum") and int(np.prod(out_shape)) >= STAGED_MIN_ELEMENTS
                and all(o.shape == out_shape for o in ops)):
            # large equal-shape elementwise calls: the pooled, chunked host pipeline
            self._ready()
            if self._stager is None:
                from ._hostpath import PluginStager
                self._stager = PluginStager(self)
            codes, masks, _ = self._stager.run(op, fmt.bits, [np.ascontiguousarray(o) for o in ops],
                                               OP_EVENTS[op], _EVENT_BIT, pow_n=int(kw.get("n", 0)))
            return codes, masks
        xs = [self.upload(o) for o in ops]
        if op == "matmul_wide" and "shift" in kw and not isinstance(kw["shift"], (int, np.integer)):
            kw = dict(kw)
            kw["shift"] = np.asarray(kw["shift"], dtype=np.int64)
        codes, cnt, fl = self.run_device(op, fmt, *xs, flags=True, **kw)
        _lib.check_counts(cnt.cpu().numpy())
        codes = codes.cpu().numpy().astype(np.int64)
        fl = fl.cpu().numpy()
        masks = {e: (fl & _EVENT_BIT[e]) != 0 for e in OP_EVENTS[op]}
        return codes, masks


def _axis(axis, ndim) -> int:
    a = int(axis)
    if a < 0:
        a += ndim
    if not 0 <= a < max(ndim, 1):
        raise SFShapeError(f"axis {axis} is out of bounds for an array of dimension {ndim}")
    return a


def _ld(T):
    """Row stride of a row-major matrix; a single row may carry any stride
    (NumPy and torch leave size-1 dimensions' strides arbitrary)."""
    return T.stride(-2) if T.shape[-2] > 1 else T.shape[-1]


def _batched(T, batch_shape, nb):
    """(…, R, C) -> a tensor whose batch entries are ``stride`` elements apart
    (0 when one matrix serves the whole batch), rows contiguous."""
    R, C = T.shape[-2], T.shape[-1]
    if T.stride(-1) != 1:
        T = T.contiguous()
    lead = tuple(T.shape[:-2])
    if all(d == 1 for d in lead):
        T2 = T.reshape(R, C) if T.is_contiguous() else T.reshape(R, C).contiguous()
        return T2, 0
    if lead == tuple(batch_shape) and T.is_contiguous():
        return T.reshape(nb, R, C), R * C
    T = T.expand(tuple(batch_shape) + (R, C)).contiguous()
    return T.reshape(nb, R, C), R * C


_registry: dict = {}


def get_device(name):
    if isinstance(name, Device):
        return name
    if name not in _registry:
        if name == "b200":
            _registry["b200"] = B200Device()
        else:
            raise SFUnsupportedError(f"unknown device {name!r}; known: host, " + ", ".join(_registry or ["b200"]))
    return _registry[name]


def register_device(device: Device) -> None:
    _registry[device.name] = device


def devices() -> tuple:
    return (HOST,) + tuple(sorted(set(_registry) | {"b200"}))
