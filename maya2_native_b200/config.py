"""Geometry of the three stages of the Maya3 decode tick.

The defaults are the benchmark geometry: a Qwen3-0.6B-class backbone, an 8-codebook depth stack (cb0 from the
backbone plus 7 depth levels, one private weight group per level) and the 8-codebook Mimi decoder.  The reference
hard-codes its depth geometry as module globals (``tts/model/depth_v2.py:45-47``, ``serve/fast_depth.py:28-29``);
here every size is a field so the production geometry (32 codebooks, shared band groups) is just another instance.
"""
from __future__ import annotations

import dataclasses
import math

N_CODES = 2048          # per-codebook vocabulary (tts/tokens.py:22)
AEOS_CLASS = N_CODES    # cb0 head class 2048 = end of audio (tts/tokens.py:23)
SAMPLE_RATE = 24000
FRAME = 1920            # PCM samples per 80 ms frame (maya3/engine.py:43)


@dataclasses.dataclass(frozen=True)
class BackboneGeom:
    """Qwen3 decoder geometry (HF Qwen3Config fields) plus the cb0 head width."""
    layers: int = 28
    hidden: int = 1024
    heads: int = 16
    kv_heads: int = 8
    head_dim: int = 128
    ffn: int = 3072
    vocab: int = 151936
    eps: float = 1e-6
    rope_theta: float = 1e6
    n_cb0: int = N_CODES + 1

    @property
    def groups(self) -> int:
        return self.heads // self.kv_heads

    @property
    def qkv_width(self) -> int:
        return (self.heads + 2 * self.kv_heads) * self.head_dim

    def kv_bytes_per_token(self, elem: int = 2) -> int:
        """K and V bytes one token adds to one seat over all layers (112 KiB at this geometry in bf16)."""
        return self.layers * 2 * self.kv_heads * self.head_dim * elem


def _default_groups(n_q: int) -> tuple:
    """Level -> weight group.  Levels 1..8 own groups 0..7; 9-16, 17-24, 25-31 share groups 8, 9, 10
    (tts/model/depth_v2.py:45).  For n_q <= 9 every level owns its group."""
    table = [None] + list(range(8)) + [8] * 8 + [9] * 8 + [10] * 7
    return tuple(table[:n_q])


@dataclasses.dataclass(frozen=True)
class DepthGeom:
    """DepthV2 geometry (tts/model/depth_v2.py:45-48,191-237)."""
    layers: int = 4
    d: int = 1024
    heads: int = 8
    ffn: int = 3072
    n_q: int = 8
    n_codes: int = N_CODES
    rank: int = 128
    d_backbone: int = 1024
    group_of_level: tuple = ()
    ln_eps: float = 1e-5

    def __post_init__(self):
        if not self.group_of_level:
            object.__setattr__(self, "group_of_level", _default_groups(self.n_q))

    @property
    def head_dim(self) -> int:
        return self.d // self.heads

    @property
    def n_groups(self) -> int:
        return max(g for g in self.group_of_level[1:]) + 1


@dataclasses.dataclass(frozen=True)
class MimiGeom:
    """HF MimiConfig decoder-side geometry (transformers MimiConfig defaults, 8 quantizers)."""
    hidden: int = 512
    n_q: int = 8
    n_semantic: int = 1
    codebook_size: int = N_CODES
    codebook_dim: int = 256
    layers: int = 8
    heads: int = 8
    ffn: int = 2048
    window: int = 250
    ring: int = 256
    ratios: tuple = (8, 6, 5, 4)
    num_filters: int = 64
    kernel: int = 7
    last_kernel: int = 3
    res_kernel: int = 3
    compress: int = 2
    rope_theta: float = 1e4
    norm_eps: float = 1e-5
    upsample_stride: int = 2

    @property
    def head_dim(self) -> int:
        return self.hidden // self.heads

    @property
    def samples_per_frame(self) -> int:
        return self.upsample_stride * math.prod(self.ratios)


@dataclasses.dataclass(frozen=True)
class Maya3Geom:
    backbone: BackboneGeom = BackboneGeom()
    depth: DepthGeom = DepthGeom()
    mimi: MimiGeom = MimiGeom()


BASELINE = Maya3Geom()

# A small geometry with the same structure, used by fast CPU tests and the golden fixtures.
TINY = Maya3Geom(
    backbone=BackboneGeom(layers=2, hidden=256, heads=4, kv_heads=2, head_dim=128, ffn=512, vocab=1000),
    depth=DepthGeom(layers=2, d=256, heads=2, ffn=512, n_q=4, rank=32, d_backbone=256),
    mimi=MimiGeom(hidden=64, n_q=4, codebook_dim=32, layers=2, heads=2, ffn=128, window=10, ring=16,
                  ratios=(4, 3), num_filters=16),
)
