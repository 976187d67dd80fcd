"""Generate tests/golden/guards_loop.npz by running the REFERENCE's own loop detector (maya3/guards.py:80-106,
loop_detect_batch) on cb0 streams of the three kinds its maya3/tests/test_guards.py uses (random, periodic with
noise, stalled tail) plus short and boundary-length streams, under the default GuardConfig and one non-default one.

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


if __name__ == "__main__":
    main()
