"""sfN formats, N = 4..16: signed fixed point Q1.(N-1).

A value is held as a signed integer code k in [-M, M], M = 2^(N-1) - 1,
worth k / 2^(N-1) (reference src/sf/_format.py:1-11, :21-110).  On the
device every width is stored as int16 codes.
"""
from __future__ import annotations

from dataclasses import dataclass
from fractions import Fraction

MIN_BITS, MAX_BITS = 4, 16


@dataclass(frozen=True)
class SFFormat:
    bits: int

    def __post_init__(self):
        if not MIN_BITS <= self.bits <= MAX_BITS:
            raise ValueError(f"sf width must be {MIN_BITS}..{MAX_BITS}, got {self.bits}")

    @property
    def name(self) -> str:
        return f"sf{self.bits}"

    @property
    def frac_bits(self) -> int:
        return self.bits - 1

    @property
    def scale(self) -> int:
        """2^(N-1): the code of one unit."""
        return 1 << (self.bits - 1)

    @property
    def max_code(self) -> int:
        return (1 << (self.bits - 1)) - 1

    @property
    def codes(self) -> int:
        return 2 * self.max_code + 1

    @property
    def max(self) -> Fraction:
        return Fraction(self.max_code, self.scale)

    @property
    def lsb(self) -> Fraction:
        return Fraction(1, self.scale)

    def __repr__(self) -> str:
        return f"SFFormat({self.name})"


FORMATS = {n: SFFormat(n) for n in range(MIN_BITS, MAX_BITS + 1)}
