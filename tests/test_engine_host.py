"""Host logic of the engine tick on CPU (no GPU): the m3_tick_run plan layout, the admission cap and the frame budget,
against the rules of maya3/engine.py:449-510 and the plan format documented at m3_tick_run."""
import numpy as np
import pytest

from maya2_native_b200.engine import FROM_FEEDBACK, TickConfig, admission_cap, frame_budget, plan_layout

ROWS = (1, 2, 4, 8, 16, 24, 32, 48, 64)
SEATS = (1, 2, 4, 8)
CTX = (256, 512, 1024)


def split(p, rb, sb):
    return p[:rb], p[rb:2 * rb], p[2 * rb:3 * rb], p[3 * rb:4 * rb], p[4 * rb:4 * rb + sb], p[4 * rb + sb:]


def test_plan_decode_and_prefill_rows():
    lengths = [10, 0, 300, 0, 0, 0]
    p, rb, sb, cb, keys = plan_layout([0, 2], [(3, np.array([5, 6, 7])), (4, np.array([9]))], lengths, ROWS, SEATS,
                                      CTX, dummy=5)
    assert (rb, sb, cb) == (8, 4, 512)            # 6 rows -> 8; 4 seats; context 301 -> 512
    slot, off, real, src, s_slot, s_row = split(p, rb, sb)
    assert list(slot) == [0, 2, 3, 3, 3, 4, 5, 5]
    assert list(off) == [0, 0, 0, 1, 2, 0, 0, 0]
    assert list(real) == [1, 1, 1, 1, 1, 1, 0, 0]
    assert list(src) == [FROM_FEEDBACK, FROM_FEEDBACK, 5, 6, 7, 9, -1, -1]
    assert list(s_slot) == [0, 2, 3, 4]
    assert list(s_row) == [0, 1, 4, 5]            # each new seat's last prompt row
    assert keys == (11 + 301) + (0 + 6) + (0 + 1) + 2   # decode len+1, prefill triangles, padding rows


def test_plan_prefill_continues_a_prefix():
    # a slot that already holds 20 positions (an eagerly prefilled head): its inline rows attend 21..23 keys
    p, rb, sb, cb, keys = plan_layout([], [(1, np.array([1, 2, 3]))], [0, 20, 0], ROWS, SEATS, CTX, dummy=2)
    assert keys == 20 * 3 + 6 + (rb - 3)
    assert cb == 256


def test_plan_padding_only_touches_the_dummy():
    p, rb, sb, cb, keys = plan_layout([], [], [0, 0, 0], ROWS, SEATS, CTX, dummy=2)
    slot, off, real, src, s_slot, _ = split(p, rb, sb)
    assert rb == 1 and sb == 1 and (slot == 2).all() and (real == 0).all() and (src == -1).all() and (s_slot == 2).all()


def test_plan_bucket_overflow_raises():
    with pytest.raises(ValueError):
        plan_layout(list(range(9)), [], [0] * 10, ROWS, SEATS, CTX, dummy=9)      # 9 seats > largest seat bucket
    with pytest.raises(ValueError):
        plan_layout([0], [], [1024], ROWS, SEATS, CTX, dummy=1)                    # context 1025 > 1024


def test_admission_cap_busy_rule():
    cfg = TickConfig(max_seats=16, max_admit_per_tick=8, busy_frac=0.75, busy_admit=4)
    assert admission_cap(0, cfg) == 8
    assert admission_cap(12, cfg) == 8            # 12 is not more than 0.75 * 16
    assert admission_cap(13, cfg) == 4


def test_frame_budget_clips_to_capacity():
    assert frame_budget(100, 500, 1024) == 500
    assert frame_budget(100, 1000, 1024) == 1024 - 100 - 2
    with pytest.raises(ValueError, match="leaves no room"):
        frame_budget(1015, 100, 1024)             # 1024 - 1015 - 2 = 7 < 8


def test_submit_caps_windows_and_voice_budget():
    """TickEngine.submit (host only): the piece's cap and prior-free cap are clipped to the frame budget
    (maya3/engine.py:405-411), suspend windows beyond the device's per-slot room are refused, and a voice prefix
    counts against the KV capacity like the reference's prompt does (maya3/engine.py:465-472)."""
    import itertools
    import types

    from maya2_native_b200.engine import TickEngine, Voice
    from maya2_native_b200.guards import GuardConfig
    eng = TickEngine.__new__(TickEngine)
    eng.cfg = TickConfig(max_seats=4, capacity=128, guards=GuardConfig(max_windows=2))
    eng.guards = types.SimpleNamespace(cfg=eng.cfg.guards)
    eng.pending, eng._rng, eng._ids = [], np.random.default_rng(0), itertools.count()
    s = eng.submit(np.arange(10), 50, cap=20, loose_cap=40, suspend=[(5, 9), (8, 12)])
    assert (s.max_frames, s.cap, s.loose_cap, s.suspend) == (50, 20, 40, ((5, 9), (8, 12)))
    s = eng.submit(np.arange(10), 50)
    assert s.cap == s.loose_cap == 50
    s = eng.submit(np.arange(10), 30, cap=80)
    assert s.cap == s.loose_cap == 30
    with pytest.raises(ValueError):
        eng.submit(np.arange(10), 50, suspend=[(1, 2), (10, 11), (20, 21)])     # three disjoint windows > 2
    v = Voice(np.arange(20), None, 20)
    s = eng.submit(np.arange(10), 200, voice=v)
    assert s.max_frames == 128 - 30 - 2 and s.voice is v
    eng.submit(np.arange(100), 10)                                           # fits without the prefix
    with pytest.raises(ValueError):
        eng.submit(np.arange(100), 10, voice=v)                              # 6 frames left: refused
    assert len(eng.pending) == 5
