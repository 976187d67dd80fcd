"""Triton-compatible counter-based uniforms (TEST INFRASTRUCTURE; see oracle/__init__.py).

The reference draws its sampling noise with Triton's ``tl.rand(seed, offset)`` (serve/fast_depth_kernels.py:320,347):
Philox4x32-10 (Salmon et al., "Parallel random numbers: as easy as 1, 2, 3", SC'11) keyed by (seed_lo, seed_hi) on the
counter (offset, 0, 0, 0); the first output word, read as int32 and folded to non-negative, times 4.6566127342e-10
(triton/language/random.py: philox_impl, randint4x, uint_to_uniform_float).
"""
import numpy as np

_ROUND_A = np.uint64(0xD2511F53)
_ROUND_B = np.uint64(0xCD9E8D57)
_KEY_A = np.uint32(0x9E3779B9)
_KEY_B = np.uint32(0xBB67AE85)
_MASK = np.uint64(0xFFFFFFFF)


def philox4x32(c0, c1, c2, c3, k0, k1, rounds=10):
    c0, c1, c2, c3 = (np.asarray(c, dtype=np.uint32) for c in (c0, c1, c2, c3))
    k0 = np.asarray(k0, dtype=np.uint32)
    k1 = np.asarray(k1, dtype=np.uint32)
    with np.errstate(over="ignore"):
        for _ in range(rounds):
            pb = _ROUND_B * c2.astype(np.uint64)
            pa = _ROUND_A * c0.astype(np.uint64)
            n0 = (pb >> np.uint64(32)).astype(np.uint32) ^ c1 ^ k0
            n2 = (pa >> np.uint64(32)).astype(np.uint32) ^ c3 ^ k1
            c1 = (pb & _MASK).astype(np.uint32)
            c3 = (pa & _MASK).astype(np.uint32)
            c0, c2 = n0, n2
            k0 = (k0 + _KEY_A).astype(np.uint32)
            k1 = (k1 + _KEY_B).astype(np.uint32)
    return c0, c1, c2, c3


def uniform(seed, offset):
    """tl.rand(seed, offset) for an int32 seed and int32 offsets: float32 in [0, 1)."""
    seed = np.asarray(seed, dtype=np.int64)
    off = np.asarray(offset, dtype=np.int64).astype(np.uint32)
    s64 = seed.astype(np.uint64)
    k0 = (s64 & _MASK).astype(np.uint32)
    k1 = ((s64 >> np.uint64(32)) & _MASK).astype(np.uint32)
    z = np.zeros_like(off)
    r0, _, _, _ = philox4x32(off, z, z, z, k0, k1)
    x = r0.view(np.int32).astype(np.int64)
    x = np.where(x < 0, -x - 1, x).astype(np.int32)
    return (x.astype(np.float32) * np.float32(4.6566127342e-10)).astype(np.float32)
