"""Seeded synthetic inputs for the hot-path workloads (host NumPy, int64 codes).

The reference publishes no datasets for this path; these generators stand in
with the shapes, sizes and value distributions of the workloads it is
measured on:

* ``chain_square``: sf16 A (n, n) @ B (n, n), codes uniform over every valid
  code, seed 0 (the 512 x 512 chain matmul).
* ``elementwise``: x, y, z of n codes, uniform, with 10% of indices forced to
  |v| >= 0.9 (add / fma saturate) and another 10% (the same indices in x, y
  and z) to |v| in [1, 127] codes (mul underflows); div's divisor has
  |b| > |a| for ~90% of pairs, b == 0 for ~1%, |b| <= |a| otherwise.
* ``wide_square``: A codes uniform in [-425, 425], B uniform over every code
  (about 1% of the 8192^3 wide outputs saturate at shift 0).
"""
from __future__ import annotations

import numpy as np


def _max_code(bits: int) -> int:
    return (1 << (bits - 1)) - 1


def chain_square(n: int = 512, seed: int = 0, bits: int = 16):
    M = _max_code(bits)
    rng = np.random.default_rng(seed)
    A = rng.integers(-M, M + 1, (n, n))
    B = rng.integers(-M, M + 1, (n, n))
    return A, B


def elementwise(n: int = 1 << 26, seed: int = 0, bits: int = 16):
    """Returns (x, y, z, d): x, y, z for add / sub / mul / fma, d the divisor
    for div(x, d)."""
    M = _max_code(bits)
    S = M + 1
    rng = np.random.default_rng(seed)
    x, y, z = (rng.integers(-M, M + 1, n) for _ in range(3))
    perm = rng.permutation(n)
    big, small = perm[: n // 10], perm[n // 10: n // 5]
    lo = -(-(9 * S) // 10)                                  # ceil(0.9 S)
    for v in (x, y, z):
        v[big] = rng.integers(lo, M + 1, big.size) * rng.choice(np.array([-1, 1]), big.size)
    small_mag = min(127, M)
    for v in (x, y, z):
        v[small] = rng.integers(1, small_mag + 1, small.size) * rng.choice(np.array([-1, 1]), small.size)
    u = rng.random(n)
    a = np.abs(x)
    sign = rng.choice(np.array([-1, 1]), n)
    # |b| uniform in (|a|, M] where possible, else in [1, |a|]
    gt = rng.integers(0, 1 << 62, n) % np.maximum(M - a, 1) + a + 1
    le = rng.integers(0, 1 << 62, n) % np.maximum(a, 1) + 1
    bm = np.where((u < 0.91) & (a < M), gt, le)
    d = np.where(u < 0.01, 0, sign * bm).astype(np.int64)
    return x.astype(np.int64), y.astype(np.int64), z.astype(np.int64), d


def wide_square(m: int = 8192, n: int = 8192, k: int = 8192, seed: int = 0, bits: int = 16,
                a_max: int = 425):
    M = _max_code(bits)
    rng = np.random.default_rng(seed)
    A = rng.integers(-a_max, a_max + 1, (m, k))
    B = rng.integers(-M, M + 1, (k, n))
    return A, B
