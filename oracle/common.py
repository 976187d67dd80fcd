"""Rounding emulation shared by the oracle (TEST INFRASTRUCTURE; see oracle/__init__.py).

The reference computes in fp32 and stores every intermediate tensor in its serving dtype.  ``Prec('bf16')``
rounds an fp32 array to the nearest bfloat16 (ties to even) at exactly the points where the reference stores a bf16
tensor; ``Prec('fp32')`` is the identity.
"""
import numpy as np


def bf16_round(x):
    """fp32 -> nearest bf16 (round half to even), returned as fp32 holding the bf16 value."""
    a = np.ascontiguousarray(x, dtype=np.float32)
    u = a.view(np.uint32)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    r = ((u + np.uint32(0x7FFF) + ((u >> 16) & np.uint32(1))) & np.uint32(0xFFFF0000)).astype(np.uint32)
    r = np.where(nan, u | np.uint32(0x00400000), r).astype(np.uint32)
    return r.view(np.float32).reshape(a.shape)


class Prec:
    def __init__(self, dtype):
        if dtype not in ("fp32", "bf16"):
            raise ValueError(f"dtype must be fp32 or bf16, got {dtype!r}")
        self.dtype = dtype

    def __call__(self, x):
        x = np.asarray(x, dtype=np.float32)
        return bf16_round(x) if self.dtype == "bf16" else x

    def mm(self, x, w):
        """Linear layer x @ w.T with fp32 accumulation, stored in the serving dtype."""
        return self(np.matmul(np.asarray(x, np.float32), np.asarray(w, np.float32).T))


def f32(x):
    return np.asarray(x, dtype=np.float32)


def softmax(x, axis=-1):
    m = np.max(x, axis=axis, keepdims=True)
    e = np.exp(x - m)
    return e / np.sum(e, axis=axis, keepdims=True)


def layer_norm(x, w, b, eps, rnd):
    """nn.LayerNorm / the reference's Triton _add_ln (serve/fast_depth_kernels.py:284-289): fp32 statistics,
    y = (x - mean) / sqrt(var + eps) * w + b, stored once in the serving dtype."""
    x = f32(x)
    mean = x.mean(-1, keepdims=True, dtype=np.float32)
    d = x - mean
    var = (d * d).mean(-1, keepdims=True, dtype=np.float32)
    return rnd(d / np.sqrt(var + np.float32(eps)) * w + b)


def gelu(x):
    """Exact (erf) GELU in fp32."""
    from scipy.special import erf
    x = f32(x)
    return f32(0.5 * x * (1.0 + erf(x / np.sqrt(2.0)).astype(np.float32)))


def silu(x):
    x = f32(x)
    return f32(x / (1.0 + np.exp(-x)))


def elu(x):
    x = f32(x)
    return f32(np.where(x > 0, x, np.expm1(np.minimum(x, 0))))
