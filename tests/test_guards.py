"""CPU: the loop-guard oracle against the reference's own loop detector (golden vectors from maya3/guards.py's
loop_detect_batch), the per-seat guard update on hand-built cb0 streams whose verdicts follow from the rules of
maya3/engine.py:571-617, and the host helpers of maya2_native_b200.guards (no GPU calls)."""
import dataclasses

import numpy as np
import pytest

from conftest import golden
from maya2_native_b200.guards import GuardConfig, merge_windows, split_code
from oracle.guards import BACKSTOP, CAP, NONE, PERIOD, STALL, GuardOracle, loop_detect


def _decode(hit):
    return 0 if hit is None else (-1 if hit == "stall" else int(hit.split(":")[1]))


@pytest.mark.parametrize("name", ["default", "alt"])
def test_loop_detect_matches_reference_vectors(name):
    z = golden("guards_loop.npz")
    stall, pw, pmin, pmax, _ = (int(v) for v in z[f"{name}_cfg"])
    thr = float(z[f"{name}_thr"])
    W, n, want = z[f"{name}_W"].astype(np.int64), z[f"{name}_n"], z[f"{name}_hit"]
    got = np.array([_decode(loop_detect(W[i], int(n[i]), stall, pw, thr, pmin, pmax)) for i in range(len(n))])
    assert (got == want).all(), np.flatnonzero(got != want)[:10]
    assert (want == -1).any() and (want > 0).any() and (want == 0).any()


def run(ora, slot, stream, stops=None):
    """Feed one seat's cb0 stream through the oracle; returns the packed code per frame."""
    out = []
    for t, c in enumerate(stream):
        stop = 0 if stops is None else stops[t]
        out.append(int(ora.step([slot], [stop], [c])[0]))
    return out


def cfg(**kw):
    return dataclasses.replace(GuardConfig(), **kw)


def test_stall_boost_then_backstop():
    ora = GuardOracle(cfg(), 2)
    ora.bind(0, cap=1000)
    codes = run(ora, 0, [5] * 60)
    v = [(c >> 8) & 0xFF for c in codes]
    # first due frame with a 32-frame stall is frame 32 (start=32, every=2): boost from there, backstop 24 frames on
    assert ora.boost_at[0] == 32 and ora.n_boost[0] == 1 and ora.aeos_bias[0] == 4.0
    assert v[:55] == [NONE] * 55 and v[55] == BACKSTOP            # frame 56 = 32 + 24
    assert codes[31] >> 16 == 1 and codes[30] >> 16 == 0


def test_loop_that_clears_removes_the_boost():
    ora = GuardOracle(cfg(), 1)
    ora.bind(0, cap=1000)
    rng = np.random.default_rng(0)
    stream = [9] * 40 + list(rng.integers(100, 2000, 40))
    codes = run(ora, 0, stream)
    assert ora.n_boost[0] == 1 and ora.boost_at[0] == -1 and ora.aeos_bias[0] == 0.0
    assert all((c >> 8) & 0xFF == NONE for c in codes)


def test_period_rule_and_stop_mode():
    ora = GuardOracle(cfg(mode="stop"), 1)
    ora.bind(0, cap=1000)
    stream = [1, 2, 3] * 30
    v = [(c >> 8) & 0xFF for c in run(ora, 0, stream)]
    assert v.index(PERIOD) == 63 and v[:63] == [NONE] * 63     # first due frame with a full 64-code window
    ora.bind(0, cap=1000)
    v = [(c >> 8) & 0xFF for c in run(ora, 0, [4] * 40)]
    assert v.index(STALL) == 31


def test_cap_precedes_the_loop_rule_and_windows_suspend_it():
    ora = GuardOracle(cfg(), 1)
    ora.bind(0, cap=32)
    v = [(c >> 8) & 0xFF for c in run(ora, 0, [5] * 32)]
    assert v[31] == CAP and ora.n_boost[0] == 0                 # frame 32 hits the cap: no loop check
    ora.bind(0, cap=1000, windows=[(20, 45), (46, 50)])
    run(ora, 0, [5] * 52)
    assert ora.boost_at[0] == 52                                # first due frame outside [20, 50]


def test_sampler_stop_passes_through_with_the_boost_count():
    ora = GuardOracle(cfg(), 1)
    ora.bind(0, cap=1000)
    run(ora, 0, [5] * 34)
    out = ora.step([0], [3], [5])
    assert out[0] == 3 | 1 << 16 and ora.frames[0] == 34        # no frame counted for a stopped seat
    out = ora.step([1], [0], [5])                              # the padding slot is left as is
    assert out[0] == 0


def test_host_helpers():
    assert merge_windows([(10, 20), (5, 9), (30, 29), (21, 25), (40, 50), (45, 60)]) == [(5, 25), (40, 60)]
    s, v, nb = split_code(np.array([3, 1 << 8 | 2 << 16, 0]))
    assert s.tolist() == [3, 0, 0] and v.tolist() == [0, 1, 0] and nb.tolist() == [0, 2, 0]
    with pytest.raises(ValueError):
        GuardConfig(mode="warn")
    with pytest.raises(ValueError):
        GuardConfig(pmax=64)
    with pytest.raises(ValueError):
        GuardConfig(hist=200)


def test_engine_delivery_decodes_guard_verdicts():
    """TickEngine._deliver on a hand-made readout (host logic only, no GPU): a sampler stop ends the seat without a
    frame; a guard verdict delivers the frame, then ends the seat with the reference's reason (maya3/engine.py:576-614);
    the boost count rides along."""
    import types
    from maya2_native_b200.engine import Seat, TickConfig, TickEngine
    eng = TickEngine.__new__(TickEngine)
    eng.cfg = TickConfig(max_seats=6, guards=GuardConfig())
    eng.guards = types.SimpleNamespace(cfg=eng.cfg.guards)
    eng.stats = {"frames": 0, "completed": 0, "ticks": 0}
    eng.active = []
    eng._early = set()
    released = []
    eng._release = released.append
    seats = [Seat(rid=i, prompt=np.zeros(3, np.int64), max_frames=50, seed=1, slot=i) for i in range(6)]
    for s in seats:
        s.cap = s.loose_cap = 50
    seats[0].cap, seats[0].frames = 10, 9          # prior cap below the loose cap -> cap_guard
    seats[4].frames = 49                           # the request's own budget -> max_frames
    seats[5].frames = 20
    hv = np.zeros((6, 2 + 4), np.int64)
    hv[0, 0] = 1 << 8
    hv[1, 0] = 2 << 8 | 1 << 16
    hv[2, 0] = 3 | 2 << 16
    hv[3, 0] = 1 << 16
    hv[4, 0] = 1 << 8
    hv[5, 0] = 4 << 8 | 1 << 16
    out = eng._deliver(seats, hv)
    assert [s.stop for s in seats] == ["cap_guard", "loop_backstop", "aeos_tau", None, "max_frames", "loop_period"]
    assert [s.frames for s in seats] == [10, 1, 0, 1, 50, 21]
    assert [s.n_boost for s in seats] == [0, 1, 2, 1, 0, 1]
    assert [o[3] is None for o in out] == [False, False, True, False, False, False]
    assert released == [seats[i] for i in (0, 1, 2, 4, 5)] and eng.active == [seats[3]]
    assert eng.stats["frames"] == 5 and eng.stats["completed"] == 5


REF_REASONS = ["", "cap", "cap_guard", "max_frames", "loop_backstop", "loop_stall", "loop_period", "aeos",
               "aeos_argmax", "aeos_tau", "aeos_hazard"]
STOPS = {1: "aeos", 2: "aeos_argmax", 3: "aeos_tau", 4: "aeos_hazard"}     # maya3/engine.py:46


@pytest.mark.parametrize("name", ["boost", "stop"])
def test_guard_oracle_matches_reference_engine_trace(name):
    """The oracle's per-seat update against the reference's own Engine._tick (maya3/engine.py:571-617, with its
    _release and _finish_piece), recorded by tests/golden/make_guards_golden.py on scripted cb0 streams: every seat's
    stop reason, frame count, boost count, boost start and AEOS bias after every tick."""
    z = golden("guards_engine.npz")
    stall, pw, pmin, pmax, start, every, backstop, hist, stop_mode = (int(v) for v in z[f"{name}_cfg"])
    thr, boost = (float(v) for v in z[f"{name}_thr"])
    gc = cfg(stall=stall, period_win=pw, pmin=pmin, pmax=pmax, start=start, every=every, backstop=backstop, hist=hist,
             mode="stop" if stop_mode else "boost", period_thr=thr, boost=boost)
    g = {k: z[f"{name}_{k}"] for k in ("bind", "cap", "loose", "maxf", "nwin", "win", "act", "stop", "cb0", "reason",
                                       "frames", "nboost", "boost_at", "bias")}
    T, S = g["act"].shape
    ora = GuardOracle(gc, S)
    caps = {}
    seen = set()
    for t in range(T):
        for s in np.flatnonzero(g["bind"][t]):
            ora.bind(s, int(g["cap"][t, s]), [tuple(w) for w in g["win"][t, s, :g["nwin"][t, s]]])
            caps[s] = (int(g["cap"][t, s]), int(g["loose"][t, s]), int(g["maxf"][t, s]))
        slots = [int(s) for s in np.flatnonzero(g["act"][t])]
        packed = ora.step(slots, [int(g["stop"][t, s]) for s in slots], [int(g["cb0"][t, s]) for s in slots])
        for s, p in zip(slots, packed):
            stop, verdict, nb = int(p) & 0xFF, (int(p) >> 8) & 0xFF, int(p) >> 16
            f = int(ora.frames[s])
            if stop:
                reason = STOPS[stop]
            elif verdict == CAP:
                cap, loose, maxf = caps[s]
                reason = "max_frames" if maxf and f >= maxf else ("cap_guard" if cap < loose else "cap")
            else:
                reason = {NONE: "", BACKSTOP: "loop_backstop", STALL: "loop_stall", PERIOD: "loop_period"}[verdict]
            assert reason == REF_REASONS[g["reason"][t, s]], (t, s)
            assert f == g["frames"][t, s] and nb == g["nboost"][t, s] == ora.n_boost[s], (t, s)
            assert ora.boost_at[s] == g["boost_at"][t, s], (t, s)
            if reason:
                ora.aeos_bias[s] = 0.0                  # the reference's _release clears the finished slot's bias
                seen.add(reason)
            assert ora.aeos_bias[s] == g["bias"][t, s], (t, s)
    want = {"cap", "cap_guard", "max_frames", "aeos", "aeos_argmax", "aeos_tau", "aeos_hazard"}
    want |= {"loop_stall", "loop_period"} if stop_mode else {"loop_backstop"}
    assert want <= seen, want - seen
