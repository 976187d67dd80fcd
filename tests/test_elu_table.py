"""The residual block's ELU table (csrc/seanet.cu, elu_bits) covers only the negative bf16 inputs with
2^-9 <= |x| < 8 and maps smaller magnitudes to x itself and larger ones to -1.  This checks that claim for every bf16
pattern outside the table, with expm1 in float64 rounded to bf16 (round to nearest even): the margins are wide
enough (2^-10 relative below the table, e^-8 < 2^-11 above it) that fp32 expm1f rounds the same way."""
import os
import re

import numpy as np

SRC = os.path.join(os.path.dirname(__file__), "..", "maya2_native_b200", "csrc", "seanet.cu")


def bf16_bits(x):
    """float64 -> bf16 bit pattern, round to nearest even (via float32, which is exact for these values' needs)."""
    f = np.asarray(x, np.float32).view(np.uint32).astype(np.uint64)
    r = (f + 0x7FFF + ((f >> 16) & 1)) >> 16
    return r.astype(np.uint32)


def test_elu_table_bounds():
    src = open(SRC).read()
    lo = int(re.search(r"kEluLo = (0x[0-9A-Fa-f]+)u", src).group(1), 16)
    hi = int(re.search(r"kEluHi = (0x[0-9A-Fa-f]+)u", src).group(1), 16)
    assert (lo, hi) == (0x3B00, 0x4100)
    mags = np.arange(0, 0x7F81, dtype=np.uint32)               # finite magnitudes, +inf included
    x = (((mags | 0x8000) << 16).astype(np.uint32)).view(np.float32).astype(np.float64)
    y = bf16_bits(np.expm1(x))
    below = mags < lo
    assert (y[below] == (mags[below] | 0x8000)).all()          # ELU(x) rounds to x
    above = mags >= hi
    assert (y[above] == 0xBF80).all()                          # ELU(x) rounds to -1
    # the table itself spans exactly the patterns where neither shortcut holds at both ends
    inside = ~below & ~above
    assert (y[inside] != (mags[inside] | 0x8000)).any() and (y[inside] != 0xBF80).any()
