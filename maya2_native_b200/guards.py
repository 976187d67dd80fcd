"""Loop guard and frame cap of the engine (maya3/guards.py:49-106, maya3/engine.py:571-617) on the device.

The reference runs them on the host after every tick's readout; here ``m3_guard_step`` runs them in the tick's
stream right after the cb0 sampler (``m3_tick_set_guard`` attaches them to ``m3_tick_run``).  This module holds the
host half: the configuration (the GuardConfig fields the rule uses), the per-slot state tensors the kernel updates,
binding a new piece to a slot (its frame cap and its suspend windows, which the reference derives from the text on
the host), and decoding the packed stop column of the readout.
"""
from __future__ import annotations

import dataclasses

import numpy as np
import torch

from . import _lib as L

VERDICTS = {1: "cap", 2: "loop_backstop", 3: "loop_stall", 4: "loop_period"}    # maya3/engine.py:586-614


@dataclasses.dataclass
class GuardConfig:
    """maya3/guards.py:49-75 (the fields of the loop rule and the cap; the duration prior and the text windows are
    computed by the caller)."""
    enabled: bool = True
    loop: bool = True
    stall: int = 32
    period_win: int = 64
    period_thr: float = 0.7
    pmin: int = 2
    pmax: int = 16
    start: int = 32
    every: int = 2
    mode: str = "boost"       # boost | stop
    boost: float = 4.0
    backstop: int = 24
    hist: int = 96
    max_windows: int = 32     # suspend windows kept per slot on the device

    def __post_init__(self):
        if self.mode not in ("boost", "stop"):
            raise ValueError(f"mode must be 'boost' or 'stop', got {self.mode!r}")
        if not (1 <= self.stall <= self.hist and 1 <= self.period_win <= self.hist <= 128):
            raise ValueError("need stall, period_win <= hist <= 128")
        if not (1 <= self.pmin and self.pmax < self.period_win and self.every >= 1):
            raise ValueError("need pmin >= 1, pmax < period_win, every >= 1")


def merge_windows(windows):
    """The union of inclusive frame windows [(a, b), ...] as sorted disjoint windows (the loop rule only asks whether
    a frame lies in any of them, so merging changes no decision)."""
    out = []
    for a, b in sorted((int(a), int(b)) for a, b in windows if int(a) <= int(b)):
        if out and a <= out[-1][1] + 1:
            out[-1] = (out[-1][0], max(out[-1][1], b))
        else:
            out.append((a, b))
    return out


def split_code(code):
    """Packed stop column (stop | verdict << 8 | n_boost << 16) -> (sampler stop code, guard verdict, n_boost)."""
    c = np.asarray(code, np.int64)
    return c & 0xFF, (c >> 8) & 0xFF, c >> 16


class DeviceGuards:
    """Per-slot guard state on the device, updated by m3_guard_step.  `aeos_bias` is the cb0 sampler's per-slot AEOS
    bias tensor (Cb0Sampler.aeos_bias), which the guard's EOS boost writes."""

    def __init__(self, cfg: GuardConfig, max_slots: int, aeos_bias: torch.Tensor):
        self.cfg = cfg
        self.max_slots = max_slots
        dev = self.device = aeos_bias.device       # the state lives beside the sampler's bias
        if aeos_bias.dtype != torch.float32 or aeos_bias.numel() < max_slots + 1:
            raise ValueError("aeos_bias must be float32 with max_slots + 1 entries")
        n = max_slots + 1
        i32 = dict(dtype=torch.int32, device=dev)
        self.frames = torch.zeros(n, **i32)
        self.cap = torch.full((n,), 2 ** 31 - 1, **i32)
        self.boost_at = torch.full((n,), -1, **i32)
        self.n_boost = torch.zeros(n, **i32)
        self.hist = torch.full((n, cfg.hist), -1, **i32)
        self.n_windows = torch.zeros(n, **i32)
        self.windows = torch.zeros(n, max(cfg.max_windows, 1), 2, **i32)
        self.aeos_bias = aeos_bias
        self.c_cfg = L.GuardConfig(int(cfg.enabled and cfg.loop), cfg.stall, cfg.period_win, float(cfg.period_thr),
                                   cfg.pmin, cfg.pmax, cfg.start, cfg.every, 0 if cfg.mode == "boost" else 1,
                                   float(cfg.boost), cfg.backstop, cfg.hist, cfg.max_windows, max_slots)
        self.c_state = L.GuardState(*[t.data_ptr() for t in (self.frames, self.cap, self.boost_at, self.n_boost,
                                                             self.hist, self.n_windows, self.windows,
                                                             self.aeos_bias)])

    @torch.inference_mode()
    def bind(self, slot: int, cap: int, windows=()):
        """A new piece on `slot` (maya3/engine.py:420-447): frame count, boost and history reset, its frame cap and
        its suspend windows (merged; more than max_windows disjoint windows is an error).  Stream-ordered writes."""
        if not 0 <= slot < self.max_slots:
            raise IndexError(slot)
        w = merge_windows(windows)
        if len(w) > self.cfg.max_windows:
            raise ValueError(f"{len(w)} disjoint suspend windows exceed max_windows={self.cfg.max_windows}")
        self.frames[slot] = 0
        self.cap[slot] = int(min(max(int(cap), 0), 2 ** 31 - 1))
        self.boost_at[slot] = -1
        self.n_boost[slot] = 0
        self.hist[slot] = -1
        self.n_windows[slot] = len(w)
        if w:
            self.windows[slot, :len(w)] = torch.tensor(w, dtype=torch.int32)
        self.aeos_bias[slot] = 0

    def step(self, slots: torch.Tensor, code: torch.Tensor, cb0: torch.Tensor, stream=None):
        """m3_guard_step on device int64 tensors: `code` (the sampler's stop codes) is packed in place."""
        n = int(slots.shape[0])
        for t in (slots, code, cb0):
            if t.dtype != torch.int64 or t.device != self.device or t.shape[0] < n or not t.is_contiguous():
                raise ValueError("slots, code and cb0 must be contiguous int64 device tensors of one length")
        L.check(L.load().m3_guard_step(self.c_cfg, self.c_state, slots.data_ptr(), code.data_ptr(), cb0.data_ptr(),
                                       n, L.stream_ptr(stream)), "m3_guard_step")


__all__ = ["GuardConfig", "DeviceGuards", "VERDICTS", "merge_windows", "split_code"]
