"""Generate the guard fixtures by running the REFERENCE's own code.

guards_loop.npz: its loop detector (maya3/guards.py:80-106, loop_detect_batch) on cb0 streams of the three kinds its
maya3/tests/test_guards.py uses (random, periodic with noise, stalled tail) plus short and boundary-length streams,
under the default GuardConfig and one non-default one.

guards_engine.npz: its engine tick (maya3/engine.py:514-630, Engine._tick, with its own _release and _finish_piece)
driven on CPU with stand-in stages -- the backbone, depth and codec return zeros and the cb0 sampler returns scripted
(stop code, cb0) pairs -- so that the per-seat guard update after the readout (:571-617) runs as the reference wrote
it: seats bound with random caps, prior-free caps, frame budgets and suspend windows, cb0 streams switching between
random, stalled and periodic segments, occasional sampler stops, new seats entering freed slots.  Recorded per tick
and slot: the stop reason, frames, boosts, the boost's start frame and the slot's AEOS bias.

    python tests/golden/make_guards_golden.py --ref /path/to/maya2-native

The reference checkout is read-only and is not needed at test time; only inputs and the reference's outputs are
stored (histories as int8: the streams use codes -1..49).  Verdicts are encoded as 0 = none, -1 = stall, p = period p.
"""
import argparse
import dataclasses
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def streams(rng, count, hist):
    Ws, ns = [], []
    for t in range(count):
        kind = t % 4
        n = int(rng.integers(0, 220)) if kind == 3 else int(rng.integers(30, 200))
        if kind == 0:
            c = rng.integers(0, 50, n)
        elif kind == 1:
            p = int(rng.integers(2, 18))
            base = rng.integers(0, 30, p)
            c = np.array([base[i % p] for i in range(n)], np.int64)
            c[rng.random(n) < rng.random() * 0.5] = rng.integers(0, 30)
        elif kind == 2:
            c = rng.integers(0, 3, n)
            c[-int(rng.integers(1, 40)):] = 7
        else:   # short streams, few symbols: stalls and periods right at the frame thresholds
            c = rng.integers(0, 2, n)
        W = np.full(hist, -1, np.int64)
        tail = c[-hist:]
        if len(tail):
            W[-len(tail):] = tail
        Ws.append(W)
        ns.append(n)
    return np.stack(Ws), np.array(ns, np.int64)


def encode(hits):
    return np.array([0 if h is None else (-1 if h == "stall" else int(h.split(":")[1])) for h in hits], np.int64)


REASONS = ["", "cap", "cap_guard", "max_frames", "loop_backstop", "loop_stall", "loop_period", "aeos", "aeos_argmax",
           "aeos_tau", "aeos_hazard"]


class Segments:
    """cb0 stream of one seat: random, stalled or periodic segments of random length."""

    def __init__(self, rng):
        self.rng, self.seg = rng, None

    def next(self):
        rng = self.rng
        if self.seg is None or self.seg["left"] == 0:
            p = int(rng.integers(2, 18))
            self.seg = {"kind": int(rng.integers(0, 3)), "left": int(rng.integers(8, 90)), "t": 0,
                        "code": int(rng.integers(0, 2048)), "base": rng.integers(0, 40, p),
                        "noise": float(rng.random() * 0.4)}
        g = self.seg
        g["left"] -= 1
        g["t"] += 1
        if g["kind"] == 0:
            return int(rng.integers(0, 2048))
        if g["kind"] == 1:
            return g["code"]
        if rng.random() < g["noise"]:
            return int(rng.integers(0, 40))
        return int(g["base"][g["t"] % len(g["base"])])


def engine_trace(G, E, gcfg, seed, n_slots=12, ticks=600, max_windows=4):
    import collections
    import threading
    import time
    import types

    import torch
    rng = np.random.default_rng(seed)
    D = 8
    eng = E.Engine.__new__(E.Engine)
    eng.cfg = types.SimpleNamespace(guards=gcfg, gap_s=0.0)
    eng.active, eng._pending, eng._cv = [], collections.deque(), threading.Condition()
    eng.device = "cpu"
    eng.feedback = torch.zeros(n_slots + 1, D)
    eng.h = torch.zeros(n_slots + 1, D)
    eng.aeos_bias = torch.zeros(n_slots + 1)
    eng.free = []
    eng.stats = {"ticks": 0, "completed": 0}
    eng.tick_ms = []
    eng._host = torch.zeros(n_slots, 2 + E.FRAME // 4, dtype=torch.int64)
    eng._evt = types.SimpleNamespace(record=lambda: None, synchronize=lambda: None)
    eng._emit = lambda req, kind, payload: None
    eng.backbone = types.SimpleNamespace(step=lambda slots, x: torch.zeros(len(slots), D), free=lambda slot: None)
    eng.depth = lambda slots, h, cb0: (torch.zeros(len(slots), 8, dtype=torch.long), torch.zeros(len(slots), D))
    eng.codec = types.SimpleNamespace(decode=lambda slots, codes: torch.zeros(len(slots), E.FRAME))
    queue, now = [], {}
    eng._admit = lambda: (queue[:], [])

    def cb0_fn(h, idx):
        sl = idx.tolist()
        return (torch.tensor([now[s][0] for s in sl], dtype=torch.long),
                torch.tensor([now[s][1] for s in sl], dtype=torch.long))
    eng._cb0 = cb0_fn

    T, S = ticks, n_slots
    z = lambda dt=np.int32: np.zeros((T, S), dt)
    out = {k: z() for k in ("cap", "loose", "maxf", "frames", "nboost", "boost_at")}
    out.update({k: z(np.int8) for k in ("bind", "act", "stop", "reason", "nwin")})
    out["cb0"] = z(np.int16)
    out["bias"] = z(np.float32)
    out["win"] = np.zeros((T, S, max_windows, 2), np.int32)
    seat_of, streams = [None] * S, [None] * S
    for t in range(T):
        queue.clear()
        for s in range(S):
            if seat_of[s] is None and rng.random() < 0.5:
                loose = int(rng.integers(60, 400))
                cap = min(loose, int(rng.integers(30, 400)))
                maxf = int(rng.integers(30, 400)) if rng.random() < 0.3 else 0
                if maxf:
                    cap = min(cap, maxf)
                wins = []
                for _ in range(int(rng.integers(0, max_windows + 1))):
                    a0 = int(rng.integers(0, 200))
                    wins.append((a0, a0 + int(rng.integers(0, 60))))
                req = types.SimpleNamespace(cancelled=False, frames=0, max_frames=maxf or None, t_first=None,
                                            t_submit=time.perf_counter(), stops=[], k=0, pieces=["x"], done=False)
                seat = E._Seat(req, s, cap, loose, 4, tuple(wins), gcfg.hist)
                queue.append(seat)
                seat_of[s], streams[s] = seat, Segments(rng)
                out["bind"][t, s], out["cap"][t, s], out["loose"][t, s], out["maxf"][t, s] = 1, cap, loose, maxf
                out["nwin"][t, s] = len(wins)
                for k, w in enumerate(wins):
                    out["win"][t, s, k] = w
        now.clear()
        for s in range(S):
            if seat_of[s] is not None:
                stop = int(rng.integers(1, 5)) if rng.random() < 0.01 else 0
                now[s] = (stop, streams[s].next())
                out["act"][t, s], out["stop"][t, s], out["cb0"][t, s] = 1, now[s][0], now[s][1]
        eng._tick()
        for s in range(S):
            seat = seat_of[s]
            if seat is None:
                continue
            out["frames"][t, s], out["nboost"][t, s] = seat.frames, seat.n_boost
            out["boost_at"][t, s] = -1 if seat.boost_at is None else seat.boost_at
            out["bias"][t, s] = float(eng.aeos_bias[s])
            if seat.req.stops:
                out["reason"][t, s] = REASONS.index(seat.req.stops[-1]["reason"])
                seat_of[s] = None
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="reference checkout (read-only)")
    a = ap.parse_args()
    sys.path.insert(0, a.ref)
    from maya3 import guards as G
    rng = np.random.default_rng(2024)
    out = {}
    alt = dataclasses.replace(G.GuardConfig(), stall=20, period_win=48, period_thr=0.6, pmin=3, pmax=10)
    for name, cfg in (("default", G.GuardConfig()), ("alt", alt)):
        W, n = streams(rng, 1500, cfg.hist)
        out[f"{name}_W"] = W.astype(np.int8)   # codes here are -1..49
        out[f"{name}_n"] = n
        out[f"{name}_hit"] = encode(G.loop_detect_batch(W, n, cfg))
        out[f"{name}_cfg"] = np.array([cfg.stall, cfg.period_win, cfg.pmin, cfg.pmax, cfg.hist], np.int64)
        out[f"{name}_thr"] = np.array(cfg.period_thr)
    np.savez_compressed(os.path.join(HERE, "guards_loop.npz"), **out)
    for name in ("default", "alt"):
        h = out[f"{name}_hit"]
        print(name, "stall", int((h == -1).sum()), "period", int((h > 0).sum()), "none", int((h == 0).sum()))

    from maya3 import engine as E
    trace = {}
    stop_cfg = dataclasses.replace(G.GuardConfig(), mode="stop", stall=20, period_win=48, period_thr=0.6, pmin=3,
                                   pmax=10, start=16, every=3)
    for name, cfg, seed in (("boost", G.GuardConfig(), 11), ("stop", stop_cfg, 12)):
        tr = engine_trace(G, E, cfg, seed)
        trace.update({f"{name}_{k}": v for k, v in tr.items()})
        trace[f"{name}_cfg"] = np.array([cfg.stall, cfg.period_win, cfg.pmin, cfg.pmax, cfg.start, cfg.every,
                                         cfg.backstop, cfg.hist, int(cfg.mode == "stop")], np.int64)
        trace[f"{name}_thr"] = np.array([cfg.period_thr, cfg.boost])
        r = tr["reason"]
        print(name, {REASONS[i]: int((r == i).sum()) for i in range(1, len(REASONS)) if (r == i).any()})
    np.savez_compressed(os.path.join(HERE, "guards_engine.npz"), **trace)


if __name__ == "__main__":
    main()
