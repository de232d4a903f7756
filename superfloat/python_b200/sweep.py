"""Exhaustive sweep of every operand pair of one width, on the GPU.

The device counterpart of the reference's exhaustive check
(tools/exhaustive.py:146-181): for an op in add / sub / mul / div and a
width N, every pair (a, b) of codes in [-M, M] is evaluated with the same
device arithmetic as the elementwise kernels.  Writing 2^32 results out is
pointless, so each a-row is folded on the device into two 64-bit digests,

    codes[a] = sum_j  uint64(code(a, b_j)) * w_j      (mod 2^64)
    flags[a] = sum_j  uint64(flags(a, b_j)) * w_j     (mod 2^64)

with b_j = j - M, w_j = splitmix64(j) and the flag bits overflow 1,
underflow 2, divide 4, invalid 8; plus the event totals.  The digest of a
sweep is the sha256 of the little-endian row digests (codes, then flags),
computed here on the host.  Rows shard across GPUs with no exchange but the
final gather.
"""
from __future__ import annotations

import hashlib

import numpy as np

from . import _lib

OPS = ("add", "sub", "mul", "div")
FLAG_BITS = {"overflow": 1, "underflow": 2, "divide": 4, "invalid": 8}


def splitmix64(x: np.ndarray) -> np.ndarray:
    """The splitmix64 output function (Steele, Lea and Flood 2014) on uint64."""
    z = np.asarray(x, dtype=np.uint64) + np.uint64(0x9E3779B97F4A7C15)
    z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
    z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
    return z ^ (z >> np.uint64(31))


def weights(bits: int) -> np.ndarray:
    M = (1 << (bits - 1)) - 1
    return splitmix64(np.arange(2 * M + 1, dtype=np.uint64))


def fold_rows(codes: np.ndarray, flags: np.ndarray, w: np.ndarray):
    """Row digests of (rows, 2M+1) code and flag arrays (the host restatement
    of what the sweep kernel accumulates)."""
    with np.errstate(over="ignore"):
        dc = (codes.astype(np.int64).astype(np.uint64) * w[None, :]).sum(axis=1, dtype=np.uint64)
        df = (flags.astype(np.uint64) * w[None, :]).sum(axis=1, dtype=np.uint64)
    return dc, df


def digest(row_codes: np.ndarray, row_flags: np.ndarray) -> str:
    h = hashlib.sha256()
    h.update(np.ascontiguousarray(row_codes, dtype="<u8").tobytes())
    h.update(np.ascontiguousarray(row_flags, dtype="<u8").tobytes())
    return h.hexdigest()


def run_device(op: str, bits: int, a_lo: int | None = None, a_hi: int | None = None, device=None, stream=None):
    """Row digests for a in [a_lo, a_hi) (default: all 2M+1 codes) on the
    current CUDA device.  Returns (row_codes, row_flags) uint64 device
    tensors and the event counts (int64 device tensor of 8)."""
    import torch
    M = (1 << (bits - 1)) - 1
    a_lo = -M if a_lo is None else a_lo
    a_hi = M + 1 if a_hi is None else a_hi
    n = max(0, a_hi - a_lo)
    dev = device or torch.device("cuda", torch.cuda.current_device())
    rc = torch.zeros(n, dtype=torch.int64, device=dev)
    rf = torch.zeros(n, dtype=torch.int64, device=dev)
    cnt = torch.zeros(_lib.N_COUNTS, dtype=torch.int64, device=dev)
    _lib.sweep(op, bits, a_lo, a_hi, rc, rf, cnt, stream)
    return rc, rf, cnt


def host_rows(rc, rf):
    """Device int64 row digests as host uint64 arrays."""
    return rc.cpu().numpy().view(np.uint64), rf.cpu().numpy().view(np.uint64)
