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
