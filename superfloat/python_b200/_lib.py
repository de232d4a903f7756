"""ctypes binding of libsfb200.so (the C ABI declared in include/sfb200.h).

The library is loaded from this package's directory; there is no fallback:
when it is missing or no sm_100 device is present every call raises
``SFDeviceError``.  Device buffers are torch tensors on the current CUDA
device (torch is the allocator and the stream owner here); the library only
sees raw pointers and a ``cudaStream_t``.
"""
from __future__ import annotations

import ctypes
import os
import threading

from ._errors import SFDeviceError, SFLaunchError, SFShapeError

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libsfb200.so")

SFB_OK, SFB_EINVAL, SFB_ECUDA, SFB_ERANGE, SFB_ENODEV = 0, -1, -2, -3, -4
F_OVERFLOW, F_UNDERFLOW, F_DIVIDE, F_INVALID, F_ACC_CLIPPED = 1, 2, 4, 8, 16
OPS = {"add": 0, "sub": 1, "mul": 2, "div": 3, "fma": 4, "neg": 5, "abs": 6, "sqrt": 7, "pow": 8}
MX = {"v4.9.2": 0, "v4.8.1": 1}
COUNT_FIELDS = ("overflow", "underflow", "divide", "invalid", "acc_clipped")
N_COUNTS = 8                       # sfb_counts: 8 x uint64

# every symbol include/sfb200.h declares: name -> (restype, argtypes)
_p, _i32, _i64 = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64
SIGNATURES = {
    "sfb_abi_version": (_i32, []),
    "sfb_last_error": (ctypes.c_char_p, []),
    "sfb_device_init": (_i32, [_i32]),
    "sfb_elementwise": (_i32, [_i32, _i32, _p, _p, _p, _p, _p, _i64, _i32, _p, _p]),
    "sfb_matmul_chain": (_i32, [_i32, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64,
                                _i64, _p, _p]),
    "sfb_linear_chain": (_i32, [_i32, _p, _p, _p, ctypes.c_double, _p, _i32, _p, _p, _p, _p, _i64, _i64, _i64,
                                _i64, _i64, _p, _p]),
    "sfb_scan": (_i32, [_p, _i32, _i64, _p, _p]),
    "sfb_quantize": (_i32, [_p, _i32, _i64, _i64, _i64, ctypes.c_double, _p, _i32, _p, _i64, _p, _p]),
    "sfb_matmul_wide_workspace": (_i64, [_i32, _i32, _i64, _i64, _i64, _i64]),
    "sfb_matmul_wide": (_i32, [_i32, _i32, _p, _p, _p, _i32, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _i64,
                               _i64, _i64, _i64, _i64, _i64, _p, _i64, _p, _p]),
    "sfb_matmul_wide_noalloc": (_i32, [_i32, _i32, _p, _p, _p, _i32, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64,
                                       _i64, _i64, _i64, _i64, _i64, _i64, _p, _p]),
    "sfb_wide_wait_limit": (_i32, [ctypes.c_uint, _i32]),
    "sfb_wide_prepared_b_bytes": (_i64, [_i32, _i32, _i64, _i64]),
    "sfb_wide_prepare_b": (_i32, [_i32, _i32, _p, _i64, _i64, _i64, _p, _i64, _p]),
    "sfb_matmul_wide_prepared": (_i32, [_i32, _i32, _p, _p, _p, _p, _i32, _p, _p, _i64, _i64, _i64, _i64, _i64,
                                        _i64, _i64, _i64, _i64, _i64, _i64, _p, _i64, _p, _p]),
    "sfb_sweep": (_i32, [_i32, _i32, _i64, _i64, _p, _p, _p]),
    "sfb_reduce_workspace": (_i64, [_i64, _i64]),
    "sfb_to_bits": (_i32, [_i32, _p, _p, _i64, _p]),
    "sfb_linear_scale_scratch": (_i64, []),
    "sfb_matmul_chain_workspace": (_i64, [_i64, _i64, _i64, _i64]),
    "sfb_matmul_chain_ws": (_i32, [_i32, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64,
                                   _p, _i64, _p, _p]),
    "sfb_linear_scale": (_i32, [_p, _i32, _i64, _i64, _i64, _i32, _i64, _i64, _i32, ctypes.c_double, ctypes.c_double,
                                _p, _p, _p, _p]),
    "sfb_linear_chain_dev": (_i32, [_i32, _p, _p, _p, _p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _p,
                                    _p]),
    "sfb_bias_codes": (_i32, [_i32, _p, _p, _p, _i64, _p, _p, _p]),
    "sfb_quantize_auto": (_i32, [_p, _i32, _i64, _i64, _i64, _p, ctypes.c_double, _i32, _p, _i64, _p, _p]),
    "sfb_from_bits": (_i32, [_i32, _p, _p, _i64, _p, _p]),
    "sfb_elementwise_signmag": (_i32, [_i32, _i32, _p, _p, _p, _p, _p, _i64, _i32, _p, _p]),
    "sfb_sum": (_i32, [_i32, _p, _i64, _i64, _i64, _p, _p, _p, _i64, _p, _p]),
    "sfb_dot": (_i32, [_i32, _p, _p, _i64, _p, _p, _p, _i64, _p, _p]),
    "sfb_matmul_wide_acc": (_i32, [_i32, _i32, _p, _p, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64, _i64, _i64,
                                   _i64, _p, _i64, _p, _p]),
    "sfb_wide_finish": (_i32, [_i32, _i32, _p, _i64, _i64, _p, _p, _p, _p, _i32, _i32, _i32, _p, _p, _p, _p, _p,
                               _p, _p]),
}

_lib = None
_lock = threading.Lock()
_ready_devices: set[int] = set()


def load(path: str = LIB_PATH):
    """Load the library and bind every declared symbol (no GPU needed)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(path):
                raise SFDeviceError(f"libsfb200.so is missing at {path}; build it with "
                                    "`python -m superfloat.python_b200.build`")
            lib = ctypes.CDLL(path)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype, fn.argtypes = res, args
            _lib = lib
    return _lib


def last_error() -> str:
    return load().sfb_last_error().decode(errors="replace")


def check(rc: int, what: str) -> None:
    if rc == SFB_OK:
        return
    msg = f"{what}: {last_error()}"
    if rc == SFB_EINVAL:
        raise SFShapeError(msg)
    if rc == SFB_ERANGE:
        raise SFLaunchError(msg)
    raise SFDeviceError(msg)


def check_counts(counts) -> None:
    """Raise if a kernel recorded a device-side failure (a bounded wait that
    ran out) in the counters' first reserved slot; ``counts`` is host data."""
    if int(counts[5]) != 0:
        raise SFDeviceError(f"a libsfb200 kernel gave up waiting on the device ({int(counts[5])} CTA(s)); "
                            "the outputs of that call are not valid")
    if int(counts[6]) != 0:
        raise SFDeviceError(f"{int(counts[6])} output(s) of a chain summed without clips left the range: the "
                            "no-saturation proof passed in was wrong")


def ensure_device(index: int) -> None:
    """sfb_device_init once per device (checks it is an sm_100 part)."""
    if index in _ready_devices:
        return
    check(load().sfb_device_init(index), "sfb_device_init")
    _ready_devices.add(index)


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(stream):
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)


def elementwise(op: str, bits: int, a, b, c, out, flags, counts, pow_n: int = 0, stream=None) -> None:
    """out = op(a, b, c) over a.numel() int16 codes (all contiguous, same length)."""
    rc = load().sfb_elementwise(OPS[op], bits, _ptr(a), _ptr(b), _ptr(c), _ptr(out), _ptr(flags),
                                a.numel(), pow_n, _ptr(counts), _stream(stream))
    check(rc, f"sf {op}")


def matmul_chain(bits, A, B, bias, out, flags, counts, batch, M, N, K, lda, ldb, sa, sb, so, stream=None):
    rc = load().sfb_matmul_chain(bits, _ptr(A), _ptr(B), _ptr(bias), _ptr(out), _ptr(flags), batch, M, N, K,
                                 lda, ldb, sa, sb, so, _ptr(counts), _stream(stream))
    check(rc, "sf matmul (chain)")


def linear_chain(bits, X, WT, bias, a, s_col, proven, y32, y64, codes, flags, counts, R, N, K, ldx, ldw,
                 stream=None):
    rc = load().sfb_linear_chain(bits, _ptr(X), _ptr(WT), _ptr(bias), float(a), _ptr(s_col), int(bool(proven)),
                                 _ptr(y32), _ptr(y64), _ptr(codes), _ptr(flags), R, N, K, ldx, ldw, _ptr(counts),
                                 _stream(stream))
    check(rc, "sf linear (chain)")


QSTATS_WORDS = 8                   # sfb_qstats: 8 x 64-bit fields
_FDT = {"float32": 0, "float64": 1}


def _fdtype(t):
    name = str(t.dtype).split(".")[-1]
    if name not in _FDT:
        raise TypeError(f"expected a float32 or float64 tensor, got {t.dtype}")
    return _FDT[name]


def scan(x, stats, stream=None):
    rc = load().sfb_scan(_ptr(x), _fdtype(x), x.numel(), _ptr(stats), _stream(stream))
    check(rc, "sf scan")


def quantize(x, rows, cols, ld, scale, row_scale, bits, codes, ldc, stats, stream=None):
    rc = load().sfb_quantize(_ptr(x), _fdtype(x), rows, cols, ld, float(scale), _ptr(row_scale), bits, _ptr(codes),
                             ldc, _ptr(stats), _stream(stream))
    check(rc, "sf quantize")


def quantize_auto(x, rows, cols, ld, scan_stats, m, bits, codes, ldc, stats, stream=None):
    rc = load().sfb_quantize_auto(_ptr(x), _fdtype(x), rows, cols, ld, _ptr(scan_stats), float(m), bits, _ptr(codes),
                                  ldc, _ptr(stats), _stream(stream))
    check(rc, "sf quantize (scale from scan)")


def chain_workspace(batch, M, N, K) -> int:
    n = load().sfb_matmul_chain_workspace(batch, M, N, K)
    if n < 0:
        check(int(n), "sf matmul (chain) workspace")
    return int(n)


def matmul_chain_ws(bits, A, B, bias, out, flags, counts, batch, M, N, K, lda, ldb, sa, sb, so, workspace,
                    stream=None):
    ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    rc = load().sfb_matmul_chain_ws(bits, _ptr(A), _ptr(B), _ptr(bias), _ptr(out), _ptr(flags), batch, M, N, K,
                                    lda, ldb, sa, sb, so, _ptr(workspace), ws_bytes, _ptr(counts), _stream(stream))
    check(rc, "sf matmul (chain)")


SCALE_RESULT_WORDS = 8              # sfb_scale_result: a, a0 (float64), 6 x int64


def linear_scale_scratch() -> int:
    return int(load().sfb_linear_scale_scratch())


def linear_scale(x, R, K, ld, bits, w_max_abs, w_max_col_l1, has_bias, need_max, a_bias, codes, result, scratch,
                 stream=None):
    rc = load().sfb_linear_scale(_ptr(x), _fdtype(x), R, K, ld, bits, int(w_max_abs), int(w_max_col_l1),
                                 int(bool(has_bias)), float(need_max), float(a_bias), _ptr(codes), _ptr(result),
                                 _ptr(scratch), _stream(stream))
    check(rc, "sf linear scale search")


def linear_chain_dev(bits, X, WT, bias, a_dev, s_col, y32, y64, counts, R, N, K, ldx, ldw, stream=None):
    rc = load().sfb_linear_chain_dev(bits, _ptr(X), _ptr(WT), _ptr(bias), _ptr(a_dev), _ptr(s_col), _ptr(y32),
                                     _ptr(y64), None, None, R, N, K, ldx, ldw, _ptr(counts), _stream(stream))
    check(rc, "sf linear (chain, device scale)")


def bias_codes(bits, b, a_dev, s_col, n, codes, n_over, stream=None):
    rc = load().sfb_bias_codes(bits, _ptr(b), _ptr(a_dev), _ptr(s_col), n, _ptr(codes), _ptr(n_over),
                               _stream(stream))
    check(rc, "sf bias codes")


def qstats_view(t):
    """Host view of one sfb_qstats held in an int64[8] tensor already on the host."""
    import numpy as np
    raw = t.numpy()
    return {"nan": int(raw[0]), "inf": int(raw[1]), "absmax": float(raw[2:3].view(np.float64)[0]),
            "overflow": int(raw[3]), "underflow": int(raw[4]), "invalid": int(raw[5]),
            "max_row_l1": int(raw[6]), "max_abs": int(raw[7])}


def wide_workspace(bits, mx, batch, M, N, K) -> int:
    n = load().sfb_matmul_wide_workspace(bits, MX[mx], batch, M, N, K)
    if n < 0:
        check(int(n), "sf matmul (wide) workspace")
    return int(n)


def to_bits(bits, codes, out, stream=None):
    rc = load().sfb_to_bits(bits, _ptr(codes), _ptr(out), codes.numel(), _stream(stream))
    check(rc, "sf to_bits")


def from_bits(bits, patterns, codes, counts, stream=None):
    rc = load().sfb_from_bits(bits, _ptr(patterns), _ptr(codes), patterns.numel(), _ptr(counts), _stream(stream))
    check(rc, "sf from_bits")


def elementwise_signmag(op, bits, a, b, c, out, flags, counts, pow_n=0, stream=None):
    rc = load().sfb_elementwise_signmag(OPS[op], bits, _ptr(a), _ptr(b), _ptr(c), _ptr(out), _ptr(flags),
                                        out.numel(), int(pow_n), _ptr(counts), _stream(stream))
    check(rc, "sf elementwise (sign-magnitude)")


def check_patterns(counts, bits) -> None:
    """ValueError when a sign-magnitude word had bits at or above N (counts host data)."""
    if int(counts[7]) != 0:
        raise ValueError(f"{int(counts[7])} bit pattern(s) do not fit in {bits} bits")


def reduce_workspace(outputs, K) -> int:
    n = load().sfb_reduce_workspace(outputs, K)
    if n < 0:
        check(int(n), "sf reduction workspace")
    return int(n)


def sum_codes(bits, x, outer, K, inner, out, flags, workspace, counts, stream=None):
    ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    rc = load().sfb_sum(bits, _ptr(x), outer, K, inner, _ptr(out), _ptr(flags), _ptr(workspace), ws_bytes,
                        _ptr(counts), _stream(stream))
    check(rc, "sf sum")


def dot(bits, a, b, n, out, flags, workspace, counts, stream=None):
    ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    rc = load().sfb_dot(bits, _ptr(a), _ptr(b), n, _ptr(out), _ptr(flags), _ptr(workspace), ws_bytes,
                        _ptr(counts), _stream(stream))
    check(rc, "sf dot")


def sweep(op, bits, a_lo, a_hi, row_digest, counts, stream=None):
    if op not in ("add", "sub", "mul", "div"):
        raise ValueError(f"the sweep covers add, sub, mul and div, not {op!r}")
    rc = load().sfb_sweep(OPS[op], bits, a_lo, a_hi, _ptr(row_digest), _ptr(counts), _stream(stream))
    check(rc, "sf sweep")


def matmul_wide_acc(bits, mx, A, B, acc, clipped, counts, M, N, K, lda, ldb, workspace, stream=None):
    ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    rc = load().sfb_matmul_wide_acc(bits, MX[mx], _ptr(A), _ptr(B), _ptr(acc), _ptr(clipped), 1, M, N, K, lda, ldb,
                                    0, 0, M * N, _ptr(workspace), ws_bytes, _ptr(counts), _stream(stream))
    check(rc, "sf matmul (wide accumulators)")


def wide_finish(bits, mx, acc, M, N, row_exp, col_exp, row_norm, col_norm, h, use_rule, shift, bias, y32, y64,
                flags, stats, counts, stream=None):
    rc = load().sfb_wide_finish(bits, MX[mx], _ptr(acc), M, N, _ptr(row_exp), _ptr(col_exp), _ptr(row_norm),
                                _ptr(col_norm), int(h), int(bool(use_rule)), int(shift), _ptr(bias), _ptr(y32),
                                _ptr(y64), _ptr(flags), _ptr(stats), _ptr(counts), _stream(stream))
    check(rc, "sf wide finish")


def wide_prepared_b_bytes(bits, mx, N, K) -> int:
    n = load().sfb_wide_prepared_b_bytes(bits, MX[mx], N, K)
    if n < 0:
        check(int(n), "sf wide prepared B size")
    return int(n)


def wide_prepare_b(bits, mx, B, N, K, ldb, prep, stream=None) -> None:
    nbytes = 0 if prep is None else prep.numel() * prep.element_size()
    check(load().sfb_wide_prepare_b(bits, MX[mx], _ptr(B), N, K, ldb, _ptr(prep), nbytes, _stream(stream)),
          "sf wide prepare B")


def matmul_wide_prepared(bits, mx, A, B, prep, shift_arr, shift, out, flags, counts, batch, M, N, K, lda, ldb, sa,
                         so, ssb, ssm, ssn, workspace, stream=None):
    ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    rc = load().sfb_matmul_wide_prepared(bits, MX[mx], _ptr(A), _ptr(B), _ptr(prep), _ptr(shift_arr), int(shift),
                                         _ptr(out), _ptr(flags), batch, M, N, K, lda, ldb, sa, so, ssb, ssm, ssn,
                                         _ptr(workspace), ws_bytes, _ptr(counts), _stream(stream))
    check(rc, "sf matmul (wide, prepared B)")


def matmul_wide(bits, mx, A, B, shift_arr, shift, out, flags, counts, batch, M, N, K, lda, ldb, sa, sb, so,
                ssb, ssm, ssn, workspace, stream=None):
    ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    rc = load().sfb_matmul_wide(bits, MX[mx], _ptr(A), _ptr(B), _ptr(shift_arr), int(shift), _ptr(out),
                                _ptr(flags), batch, M, N, K, lda, ldb, sa, sb, so, ssb, ssm, ssn,
                                _ptr(workspace), ws_bytes, _ptr(counts), _stream(stream))
    check(rc, "sf matmul (wide)")
