"""GPU parity of the device loop guard and frame cap (m3_guard_step) against the CPU oracle (oracle/guards.py, whose
loop rule is pinned to the reference's loop_detect_batch by tests/test_guards.py).  Integer work: bit-exact.

Standalone: many seats over hundreds of ticks with cb0 streams that switch between random, stalled and periodic
segments (the stream kinds of the reference's maya3/tests/test_guards.py), occasional sampler stops, random caps and
suspend windows, seats rebound when they finish, the padding slot in the batch; every tick's packed codes and the
final per-slot state must equal the oracle's.  Through the tick: TickEngine with guards on, teacher-forced -- the
oracle replays each tick on the device's own sampler stop codes and cb0 samples and must produce the readout's
packed stop column, and seats must finish with the reasons the verdicts name."""
import dataclasses

import numpy as np
import pytest
import torch

from maya2_native_b200 import weights as WG
from maya2_native_b200.config import TINY
from maya2_native_b200.engine import TickConfig, TickEngine
from maya2_native_b200.guards import DeviceGuards, GuardConfig, merge_windows, split_code
from oracle.guards import GuardOracle

pytestmark = pytest.mark.gpu


class Streams:
    """Per-slot cb0 generator switching between random, stalled and periodic segments."""

    def __init__(self, rng, n):
        self.rng, self.state = rng, [None] * n

    def next(self, slot):
        st, rng = self.state[slot], self.rng
        if st is None or st["left"] == 0:
            kind = int(rng.integers(0, 3))
            p = int(rng.integers(2, 18))
            st = self.state[slot] = {"kind": kind, "left": int(rng.integers(8, 90)), "t": 0,
                                     "code": int(rng.integers(0, 2048)), "base": rng.integers(0, 40, p),
                                     "noise": float(rng.random() * 0.4)}
        st["left"] -= 1
        st["t"] += 1
        if st["kind"] == 0:
            return int(rng.integers(0, 2048))
        if st["kind"] == 1:
            return st["code"]
        if rng.random() < st["noise"]:
            return int(rng.integers(0, 40))
        return int(st["base"][st["t"] % len(st["base"])])


def windows(rng):
    out = []
    for _ in range(int(rng.integers(0, 4))):
        a = int(rng.integers(0, 200))
        out.append((a, a + int(rng.integers(0, 60))))
    return out


@pytest.mark.parametrize("gcfg", [
    GuardConfig(),
    GuardConfig(mode="stop"),
    GuardConfig(stall=20, period_win=48, period_thr=0.6, pmin=3, pmax=10, start=16, every=3, backstop=9, hist=64,
                max_windows=4),
], ids=["boost", "stop", "alt"])
def test_guard_step_matches_oracle(cuda, gcfg):
    rng = np.random.default_rng(5)
    S, ticks = 96, 420
    bias = torch.zeros(S + 1, device=cuda, dtype=torch.float32)
    dev = DeviceGuards(gcfg, S, bias)
    ora = GuardOracle(gcfg, S)
    gen = Streams(rng, S)

    def bind(slot):
        cap = int(rng.integers(20, 400))
        w = merge_windows(windows(rng))[:gcfg.max_windows]
        dev.bind(slot, cap, w)
        ora.bind(slot, cap, w)
        gen.state[slot] = None

    for s in range(S):
        bind(s)
    verdicts = np.zeros(5, np.int64)
    for t in range(ticks):
        slots = [int(s) for s in rng.permutation(S)[:int(rng.integers(S // 2, S + 1))]]
        slots += [S] * int(rng.integers(0, 3))                     # padding seats
        stops = [int(rng.integers(1, 5)) if rng.random() < 0.01 else 0 for _ in slots]
        cb0 = [gen.next(s) if s < S else 0 for s in slots]
        st = torch.tensor(slots, dtype=torch.int64, device=cuda)
        code = torch.tensor(stops, dtype=torch.int64, device=cuda)
        c0 = torch.tensor(cb0, dtype=torch.int64, device=cuda)
        dev.step(st, code, c0)
        want = ora.step(slots, stops, cb0)
        got = code.cpu().numpy()
        assert (got == want).all(), (t, np.flatnonzero(got != want)[:5])
        stop, verdict, _ = split_code(got)
        for s, sc, v in zip(slots, stop, verdict):
            if s < S and (sc or v):
                verdicts[v] += 1
                bind(s)
    torch.cuda.synchronize()
    assert (dev.frames[:S].cpu().numpy() == ora.frames).all()
    assert (dev.boost_at[:S].cpu().numpy() == ora.boost_at).all()
    assert (dev.n_boost[:S].cpu().numpy() == ora.n_boost).all()
    assert (bias[:S].cpu().numpy() == ora.aeos_bias).all()
    ring = dev.hist[:S].cpu().numpy()
    H = gcfg.hist
    for s in range(S):
        f = int(ora.frames[s])
        m = min(f, H)
        got = [ring[s, (k - 1) % H] for k in range(f - m + 1, f + 1)]
        assert got == ora.hist[s, H - m:].tolist(), s
    # every verdict kind the configuration can produce occurred
    assert verdicts[1] > 0
    if gcfg.mode == "boost":
        assert verdicts[2] > 0 and ora.n_boost.sum() + verdicts[2] > 0
    else:
        assert verdicts[3] > 0 and verdicts[4] > 0


def test_guards_through_the_tick(cuda):
    """Guards attached to m3_tick_run: with period_thr = 0 every seat 'loops' as soon as the period window is full,
    so the EOS boost and the backstop run through the tick; one seat has a short cap.  The oracle, fed each tick the
    device's sampler stop codes and cb0 samples, must reproduce the readout's packed stop column."""
    W = WG.generate(WG.all_shapes(TINY))
    g = GuardConfig(stall=8, period_win=16, period_thr=0.0, pmin=2, pmax=4, start=12, every=2, backstop=6, hist=16)
    cfg = TickConfig(max_seats=3, capacity=256, max_inline_rows=16, min_frames=2, guards=g)
    eng = TickEngine(TINY, W, cfg, device=cuda)
    ora = GuardOracle(g, 3)
    rng = np.random.default_rng(3)
    reqs = [eng.submit(rng.integers(0, TINY.backbone.vocab, 6), 60, seed=21, cap=10),
            eng.submit(rng.integers(0, TINY.backbone.vocab, 6), 60, seed=22, suspend=[(14, 20)]),
            eng.submit(rng.integers(0, TINY.backbone.vocab, 6), 60, seed=23),
            eng.submit(rng.integers(0, TINY.backbone.vocab, 6), 60, seed=24)]
    seen = set()
    for _ in range(120):
        out = eng.tick()
        if not out:
            break
        packed = eng.last_readout()[:len(out), 0].copy()
        for s, *_ in out:
            if id(s) not in seen:
                seen.add(id(s))
                ora.bind(s.slot, s.cap, merge_windows(s.suspend))
        stop = [int(p) & 0xFF for p in packed]
        cb0 = [int(c) for _, _, c, _ in out]
        want = ora.step([s.slot for s, *_ in out], stop, cb0)
        assert (packed == want).all(), (packed, want)
    assert all(r.stop is not None for r in reqs), [r.stop for r in reqs]
    a, b = reqs[0], reqs[1]
    assert a.stop in ("cap_guard", "aeos", "aeos_argmax", "aeos_tau", "aeos_hazard")
    if a.stop == "cap_guard":
        assert a.frames == 10
    assert {r.stop for r in reqs} <= {"cap_guard", "loop_backstop", "aeos", "aeos_argmax", "aeos_tau", "aeos_hazard"}
    if b.stop == "loop_backstop":
        assert b.frames == 22 + 6 and b.n_boost == 1          # suspended on 14..20: first due frame 22
    assert eng.device_status() == 0
    eng.close()
