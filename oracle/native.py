"""ctypes access to the compiled oracles (test infrastructure).

* ``oracle/_build/liboracle.so``: this repo's C restatement (``oracle.c``).
* ``oracle/_ref/libmx_ref.so``: the reference's own C accumulator
  (src/sf/_fastmx.py:41-85), compiled from the reference tree by
  ``oracle/build_ref.py``; absent when the reference was not available at
  build time.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from concurrent.futures import ThreadPoolExecutor

import numpy as np

from . import sfref

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "_build", "liboracle.so")
REF_LIB = os.path.join(HERE, "_ref", "libmx_ref.so")

_lib = None
_ref = None


def build() -> str:
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB):
            build()
        L = ctypes.CDLL(LIB)
        p, i64, i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
        L.orc_matmul_chain.argtypes = [i64, i64, i32, p, p, i64, i64, i64, p, p, p]
        L.orc_matmul_chain.restype = None
        L.orc_wide_acc.argtypes = [i64, i64, p, p, p, p, i64, i64, i64, i32, i32, i64, i32, i64, i64, p, p]
        L.orc_wide_acc.restype = None
        _lib = L
    return _lib


def _c64(x):
    return np.ascontiguousarray(x, dtype=np.int64)


def _rows(fn, M, threads=None):
    """Run fn(r0, r1) over row blocks in threads (the C calls release the GIL)."""
    nt = max(1, min(threads or os.cpu_count() or 1, M))
    cuts = np.linspace(0, M, nt + 1).astype(int)
    if nt == 1:
        fn(0, M)
        return
    with ThreadPoolExecutor(nt) as ex:
        list(ex.map(lambda i: fn(int(cuts[i]), int(cuts[i + 1])), range(nt)))


def matmul_chain(bits, A, B):
    """2-D chain matmul in C; same results as ``sfref.matmul_chain``."""
    A, B = _c64(A), _c64(B)
    M, K = A.shape
    N = B.shape[1]
    out = np.empty((M, N), np.int64)
    ov = np.empty((M, N), np.uint8)
    un = np.empty((M, N), np.uint8)
    L = lib()
    _rows(lambda r0, r1: L.orc_matmul_chain(r0, r1, bits, A.ctypes.data, B.ctypes.data, M, N, K,
                                            out.ctypes.data, ov.ctypes.data, un.ctypes.data), M)
    return out, {"overflow": ov.astype(bool), "underflow": un.astype(bool)}


def wide_acc(bits, A, B, mx=sfref.MX_DEFAULT):
    """2-D wide accumulators in C; same results as ``sfref.wide_acc``."""
    A, B = _c64(A), _c64(B)
    blk = sfref.mx_block(bits)
    u = sfref.MX_UNITS[mx][blk]
    M, K = A.shape
    N = B.shape[1]
    am, bm = _c64(sfref.mx_mags(bits, A)), _c64(sfref.mx_mags(bits, B))
    an = np.ascontiguousarray(A < 0, dtype=np.uint8)
    bn = np.ascontiguousarray(B < 0, dtype=np.uint8)
    acc = np.empty((M, N), np.int64)
    clip = np.empty((M, N), np.uint8)
    lo, hi = -(1 << (u["W"] - 1)), (1 << (u["W"] - 1)) - 1
    L = lib()
    _rows(lambda r0, r1: L.orc_wide_acc(r0, r1, am.ctypes.data, an.ctypes.data, bm.ctypes.data,
                                        bn.ctypes.data, M, N, K, int(blk == 16), int(u["tk"] or 1),
                                        int(u["comp"] or 0), int(u["F"]), lo, hi, acc.ctypes.data,
                                        clip.ctypes.data), M)
    return acc, clip.astype(bool), u["F"]


# --- the reference's own C accumulator ---------------------------------------------------

def ref_available() -> bool:
    return os.path.exists(REF_LIB)


def ref_lib():
    global _ref
    if _ref is None:
        if not ref_available():
            raise FileNotFoundError(f"{REF_LIB} was not built (python oracle/build_ref.py)")
        L = ctypes.CDLL(REF_LIB)
        i64, i32, p = ctypes.c_int64, ctypes.c_int32, ctypes.c_void_p
        # the reference's signature (src/sf/_fastmx.py:46-51, :139-140)
        L.mx_acc.argtypes = [i64, i64, i64, i64, p, p, p, p, i32, i32, i32, i32, p, i64, i64, p, p]
        L.mx_acc.restype = None
        _ref = L
    return _ref


def dropped_columns(tk: int) -> np.ndarray:
    """C[x][y] = sum over i < tk with bit i of x set of (y << i) mod 2^tk
    (src/sf/_fastmx.py:150-161): the table the reference's C loop reads."""
    x = np.arange(1 << tk, dtype=np.int64)[:, None]
    y = np.arange(1 << tk, dtype=np.int64)[None, :]
    t = np.zeros((1 << tk, 1 << tk), np.int64)
    for i in range(tk):
        t += ((x >> i) & 1) * ((y << i) & ((1 << tk) - 1))
    return np.ascontiguousarray(t, dtype=np.int32)


def ref_wide_acc(bits, A, B, mx=sfref.MX_DEFAULT, threads=None):
    """The reference's C ``mx_acc`` over row blocks in ``threads`` threads, with
    its operand preparation restated (src/sf/_fastmx.py:168-198)."""
    L = ref_lib()
    A, B = _c64(A), _c64(B)
    blk = sfref.mx_block(bits)
    u = sfref.MX_UNITS[mx][blk]
    M, K = A.shape
    N = B.shape[1]
    am = np.ascontiguousarray(sfref.mx_mags(bits, A), dtype=np.int32)
    an = -np.ascontiguousarray(A < 0, dtype=np.int32)
    bmT = np.ascontiguousarray(sfref.mx_mags(bits, B).T, dtype=np.uint16)
    bnT = np.negative(np.ascontiguousarray((B < 0).T, dtype=np.int8))
    acc = np.empty((M, N), np.int64)
    clip = np.empty((M, N), np.uint8)
    tk = int(u["tk"]) if blk == 16 else 1
    C = dropped_columns(tk)
    comp = int(u["comp"]) if blk == 16 else 0
    sh = 30 - int(u["F"]) if blk == 16 else 0
    lo, hi = -(1 << (u["W"] - 1)), (1 << (u["W"] - 1)) - 1
    args = (K, N, am.ctypes.data, an.ctypes.data, bmT.ctypes.data, bnT.ctypes.data, int(blk == 16),
            comp, sh, tk, C.ctypes.data, lo, hi, acc.ctypes.data, clip.ctypes.data)
    _rows(lambda r0, r1: L.mx_acc(r0, r1, *args), M, threads)
    return acc, clip.astype(bool), u["F"]
