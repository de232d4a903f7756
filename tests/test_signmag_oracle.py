"""The oracle's sign-magnitude words against the reference's format tables:
the table of every code, rebuilt from the oracle, has the reference's sha256
at every width; from_bits inverts it and reads the sign-only word as 0."""
import hashlib

import numpy as np
import pytest

from conftest import golden
from oracle import sfref


@pytest.mark.parametrize("bits", range(4, 17))
def test_table_digest(bits):
    M, S = sfref.consts(bits)
    k = np.arange(-M, M + 1)
    w = sfref.to_bits(bits, k)
    width = (bits + 3) // 4
    table = "".join(f"{int(c)}\t{int(x):0{width}x}\t{float(int(c) / S)!r}\n" for c, x in zip(k, w))
    assert hashlib.sha256(table.encode()).hexdigest() == golden("format_tables.json")["sha256"][f"sf{bits}"]
    back, fits = sfref.from_bits(bits, w)
    assert (back == k).all() and fits.all()
    z, _ = sfref.from_bits(bits, np.array([1 << (bits - 1)]))
    assert int(z[0]) == 0
