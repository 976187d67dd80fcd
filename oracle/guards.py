"""CPU oracle of the engine's loop guard and frame cap.  TEST INFRASTRUCTURE ONLY: imported by tests/, never by the
product path.

Restates, per seat and in plain numpy:
  * loop_detect  -- maya3/guards.py:80-106 (loop_detect_batch: a `stall`-frame stall, else the smallest period p in
                    pmin..pmax with c[t] == c[t-p] on >= period_thr of the last period_win codes; nothing before
                    max(12, stall) frames, no period before max(12, stall, period_win) frames);
  * GuardOracle  -- the per-seat update after the readout, maya3/engine.py:571-617: a seat that delivered a frame
                    counts it and shifts its cb0 into a right-aligned history; at its cap it finishes; otherwise on
                    frames >= start with frames % every == 0 outside its suspend windows the loop rule runs, and a
                    hit sets the EOS boost (boost mode; a loop persisting `backstop` frames past the boost finishes
                    the seat) or finishes it at once (stop mode); a cleared loop removes the boost.

Pinning (both fixtures made by tests/golden/make_guards_golden.py running the reference's own code): loop_detect
against guards_loop.npz, the reference's loop_detect_batch on the stream kinds of its maya3/tests/test_guards.py;
GuardOracle against guards_engine.npz, traces of the reference's Engine._tick (maya3/engine.py:514-630) driven on CPU
with stand-in stages and scripted cb0 streams -- every seat's stop reason, frames, boosts and AEOS bias per tick.
Outputs use the C ABI's packing (m3_guard_step): stop | verdict << 8 | n_boost << 16.
"""
from __future__ import annotations

import numpy as np

NONE, CAP, BACKSTOP, STALL, PERIOD = 0, 1, 2, 3, 4


def loop_detect(c, n, stall=32, period_win=64, period_thr=0.7, pmin=2, pmax=16):
    """One seat: c = its cb0 history, newest last (any length >= the windows used), n = frames generated.
    Returns None, "stall" or "period:<p>" (maya3/guards.py:80-106)."""
    c = np.asarray(c)
    if n < max(12, stall):
        return None
    tail = c[-stall:]
    if (tail == tail[0]).all():
        return "stall"
    if n >= max(12, stall, period_win):
        w = c[-period_win:]
        for p in range(pmin, pmax + 1):
            if (w[p:] == w[:-p]).mean() >= period_thr:
                return f"period:{p}"
    return None


class GuardOracle:
    """Per-slot guard state and its update, mirroring m3_guard_step.  cfg: any object with the fields of
    maya3/guards.py:49-75 GuardConfig used here (loop, stall, period_win, period_thr, pmin, pmax, start, every, mode,
    boost, backstop, hist)."""

    def __init__(self, cfg, max_slots):
        self.cfg = cfg
        self.max_slots = max_slots
        self.frames = np.zeros(max_slots, np.int64)
        self.cap = np.zeros(max_slots, np.int64)
        self.boost_at = np.full(max_slots, -1, np.int64)
        self.n_boost = np.zeros(max_slots, np.int64)
        self.hist = np.full((max_slots, cfg.hist), -1, np.int64)
        self.windows = [() for _ in range(max_slots)]
        self.aeos_bias = np.zeros(max_slots, np.float32)

    def bind(self, slot, cap, windows=()):
        """maya3/engine.py:420-447 (_bind / _Seat.__init__): a new piece on the slot."""
        self.frames[slot] = 0
        self.cap[slot] = cap
        self.boost_at[slot] = -1
        self.n_boost[slot] = 0
        self.hist[slot] = -1
        self.windows[slot] = tuple(windows)
        self.aeos_bias[slot] = 0

    def step(self, slots, code, cb0):
        """One tick's update for the seats on `slots` given the sampler's stop codes and cb0 samples; returns the
        packed codes.  Seats on the padding slot (>= max_slots) are returned unchanged."""
        g = self.cfg
        out = np.array(code, np.int64).copy()
        for i, (slot, stop, c0) in enumerate(zip(slots, code, cb0)):
            slot = int(slot)
            if not 0 <= slot < self.max_slots:
                continue
            if stop:                                            # engine.py:576-578
                out[i] = int(stop) | int(self.n_boost[slot]) << 16
                continue
            self.frames[slot] += 1                              # :579
            f = int(self.frames[slot])
            self.hist[slot, :-1] = self.hist[slot, 1:]          # :584-585
            self.hist[slot, -1] = int(c0)
            verdict = NONE
            if f >= self.cap[slot]:                             # :586-593
                verdict = CAP
            elif g.loop and f >= g.start and f % g.every == 0 and \
                    not any(a <= f <= b for a, b in self.windows[slot]):   # :594-596
                hit = loop_detect(self.hist[slot], f, g.stall, g.period_win, g.period_thr, g.pmin, g.pmax)
                if hit is not None and g.mode == "boost":       # :606-612
                    if self.boost_at[slot] < 0:
                        self.boost_at[slot] = f
                        self.n_boost[slot] += 1
                        self.aeos_bias[slot] = g.boost
                    if f - self.boost_at[slot] >= g.backstop:
                        verdict = BACKSTOP
                elif hit is not None:                           # :613-614
                    verdict = STALL if hit == "stall" else PERIOD
                elif self.boost_at[slot] >= 0:                  # :615-617
                    self.aeos_bias[slot] = 0.0
                    self.boost_at[slot] = -1
            out[i] = verdict << 8 | int(self.n_boost[slot]) << 16
        return out


__all__ = ["NONE", "CAP", "BACKSTOP", "STALL", "PERIOD", "loop_detect", "GuardOracle"]
