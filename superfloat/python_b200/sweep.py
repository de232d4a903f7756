"""Exhaustive sweep of every operand pair of one width, on the GPU.

The device counterpart of the reference's exhaustive check
(tools/exhaustive.py:146-181): for an op in add / sub / mul / div and a
width N, every pair (a, b) of codes in [-M, M] is evaluated with the same
device arithmetic as the elementwise kernels.  Writing 2^32 results out is
pointless, so each a-row is folded on the device into one 32-bit digest,

    digest[a] = sum_j  ((code(a, b_j) + M) | flags(a, b_j) << 16) * w_j      (mod 2^32)

with b_j = j - M, w_j = (the low word of splitmix64(j)) | 1 and the flag
bits overflow 1, underflow 2, divide 4, invalid 8; plus the event totals.
The weights are odd, so one wrong code or flag (a nonzero change below 2^20
of one term) always changes the digest; several cancel with probability
about 2^-32.  The digest of a sweep is the sha256 of the little-endian row
digests, computed here on the host.  Rows shard across GPUs with no exchange
but the final gather.
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
    """w_j, j = 0 .. 2M: the low word of splitmix64(j), made odd (uint64 holding 32 bits)."""
    M = (1 << (bits - 1)) - 1
    return (splitmix64(np.arange(2 * M + 1, dtype=np.uint64)) & np.uint64(0xFFFFFFFF)) | np.uint64(1)


def fold_rows(codes: np.ndarray, flags: np.ndarray, w: np.ndarray, bits: int) -> np.ndarray:
    """Row digests (uint32) of (rows, 2M+1) code and flag arrays: the host
    restatement of what the sweep kernel accumulates."""
    M = (1 << (bits - 1)) - 1
    word = (codes.astype(np.int64) + M).astype(np.uint64) | (flags.astype(np.uint64) << np.uint64(16))
    with np.errstate(over="ignore"):
        d = (word * w[None, :]).sum(axis=1, dtype=np.uint64)
    return (d & np.uint64(0xFFFFFFFF)).astype(np.uint32)


def digest(row_digests: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(row_digests, dtype="<u4").tobytes()).hexdigest()


def run_device(op: str, bits: int, a_lo: int | None = None, a_hi: int | None = None, device=None, stream=None):
    """Row digests for a in [a_lo, a_hi) (default: all 2M+1 codes) on the
    current CUDA device.  Returns the row digests (int32 device tensor
    holding the uint32 words) and the event counts (int64 device tensor of 8)."""
    import torch
    M = (1 << (bits - 1)) - 1
    a_lo = -M if a_lo is None else a_lo
    a_hi = M + 1 if a_hi is None else a_hi
    n = max(0, a_hi - a_lo)
    dev = device or torch.device("cuda", torch.cuda.current_device())
    rd = torch.zeros(n, dtype=torch.int32, device=dev)
    cnt = torch.zeros(_lib.N_COUNTS, dtype=torch.int64, device=dev)
    _lib.sweep(op, bits, a_lo, a_hi, rd, cnt, stream)
    return rd, cnt


def host_rows(rd) -> np.ndarray:
    """Device row digests as a host uint32 array."""
    return rd.cpu().numpy().view(np.uint32)
