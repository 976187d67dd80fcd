"""Swapping the native serve objects into the reference's own engine (maya3/engine.py).

``build_fast(engine)`` is ``Engine._build_fast`` (maya3/engine.py:181-234) with this package's ``StaticBackbone``,
``FastDepth``, ``StaticMimi`` and ``Cb0Sampler`` in place of serve/fast_backbone.py, serve/fast_depth.py,
serve/fast_codec.py and the engine's eager ``_cb0`` (maya3/engine.py:652-694).  It sets every attribute the
reference's method sets -- bucket ladders, the three serve objects, the hidden / feedback buffers, the per-slot
sampler tensors (here the sampler's own, so the engine's ``_bind`` writes them in place), the seed stream, free
list, pinned readout buffer and event -- and points the engine's ``_cb0`` at the sampler.  A maintainer calls it from
``Engine._build_fast``; nothing else in the engine changes.
"""
from __future__ import annotations

import types

import torch

from .backbone import StaticBackbone
from .codec import StaticMimi
from .depth import FastDepth
from .sampler import Cb0Sampler

BUCKETS = (1, 2, 4, 8, 16, 24, 32, 48, 64, 80, 96, 112, 128, 160, 192, 224, 256)                 # maya3/engine.py:44
ROW_BUCKETS = (1, 2, 4, 8, 16, 24, 32, 48, 64, 80, 96, 112, 128, 160, 192, 224, 256, 320, 384, 448, 512)  # :45
FRAME = 1920                                                                                      # maya3/engine.py:43
SLOT_TENSORS = ("frames_t", "min_t", "hazard_t", "aeos_bias", "temp_t", "topk_t", "topp_t", "rep_t", "seed_t",
                "ctr_t", "hist_t")


def build_fast(engine) -> None:
    """Engine._build_fast on the native objects (maya3/engine.py:181-234); `engine` is a reference Engine whose
    model, mimi, cfg and device are set."""
    import random

    cfg, dev = engine.cfg, engine.device
    if cfg.depth_dtype != "bf16":
        raise ValueError("the native depth stack serves bf16 only (EngineConfig.depth_dtype='bf16')")
    n = cfg.max_seats
    buckets = tuple(b for b in BUCKETS if b < n) + (next(b for b in BUCKETS if b >= n),)
    rows = tuple(b for b in ROW_BUCKETS if b <= buckets[-1] + cfg.max_inline_rows)
    rows = rows + tuple(b for b in ROW_BUCKETS if b > rows[-1])[:1]
    engine.buckets, engine.row_buckets, engine.max_rows = buckets, rows, rows[-1]
    ctx = tuple(c for c in (256, 512, 768, 1024, 1536, 2048, 3072) if c < cfg.capacity) + (cfg.capacity,)
    engine.backbone = StaticBackbone(engine.model.backbone, n, capacity=cfg.capacity, batch_buckets=rows,
                                     ctx_buckets=ctx, attention="triton", use_graphs=cfg.use_graphs,
                                     fuse_proj=cfg.fuse_proj, fused_norm=cfg.fused_norm, fuse_rope=cfg.fuse_rope,
                                     device=dev)
    engine.depth = FastDepth(engine.model, n, dtype=torch.bfloat16, batch_buckets=buckets, seed=cfg.seed + 1,
                             temp=cfg.temp, top_k=cfg.top_k, compile=cfg.compile_depth, fused=cfg.fused_depth,
                             device=dev)
    engine.codec = StaticMimi(engine.mimi, n, batch_buckets=buckets, device=dev)
    m = n + 1
    D = engine.model.backbone.d_model
    engine.h = torch.zeros(m, D, device=dev, dtype=torch.bfloat16)
    engine.feedback = torch.zeros_like(engine.h)
    sampler = Cb0Sampler(engine.model.backbone.cb0_head.weight, n, max_rows=buckets[-1], temp=cfg.cb0_temp,
                         top_k=cfg.cb0_top_k, top_p=cfg.cb0_top_p, rep=cfg.cb0_rep, rep_win=cfg.cb0_rep_win,
                         device=dev)
    engine.sampler = sampler
    for name in SLOT_TENSORS:
        setattr(engine, name, getattr(sampler, name))
    engine._seed_rng = random.Random(cfg.seed)
    engine.generator = torch.Generator(device=dev).manual_seed(cfg.seed)
    engine.free = list(range(n))[::-1]
    engine.active = []
    engine._any_rep = False
    engine._any_top_p = cfg.cb0_top_p < 1.0
    engine._host = torch.empty(n, 2 + FRAME // 4, dtype=torch.int64).pin_memory()
    engine._evt = torch.cuda.Event()
    engine.warm = False

    def _cb0(self, h, idx):
        # the engine's host flags (_any_rep, _any_top_p; set by its _bind) select the same sampler branches
        self.sampler.any_rep = bool(self._any_rep)
        self.sampler.any_top_p = bool(self._any_top_p)
        return self.sampler(h, idx)
    engine._cb0 = types.MethodType(_cb0, engine)
