"""Binding a request to a slot (maya3/engine.py:420-447 Engine._bind) through the single m3_slot_reset launch: every
per-slot field the reference's bind writes holds the request's value afterwards, whatever the slot held before, and no
other slot changes; the entry point rejects a slot outside [0, max_slots) and a misaligned speaker constant."""
import numpy as np
import pytest
import torch

from maya2_native_b200 import _lib as L
from maya2_native_b200 import weights as WG
from maya2_native_b200.config import TINY
from maya2_native_b200.engine import TickConfig, TickEngine

pytestmark = pytest.mark.gpu


def fields(eng):
    c, d = eng.cb0, eng.depth
    return {"frames": c.frames_t, "min": c.min_t, "hazard": c.hazard_t, "aeos": c.aeos_bias, "seed": c.seed_t,
            "ctr": c.ctr_t, "hist": c.hist_t, "temp": c.temp_t, "top_k": c.topk_t, "top_p": c.topp_t, "rep": c.rep_t,
            "row_seed": d.row_seed, "row_ctr": d.row_ctr, "cross": d.cross_const, "lengths": eng.backbone.lengths}


def snapshot(eng):
    torch.cuda.synchronize()
    return {k: v.detach().cpu().clone() for k, v in fields(eng).items()}


def dirty(eng):
    """Garbage in every per-slot field of every slot, as a finished request leaves it."""
    with torch.inference_mode():
        for k, v in fields(eng).items():
            if v.dtype.is_floating_point:
                v.copy_(torch.randn_like(v.float()).to(v.dtype) * 3 + 7)
            else:
                v.copy_(torch.randint_like(v, 1, 1000))


def expected(eng, s):
    cfg, sp = eng.cfg, s.sampling
    rep = sp["repetition_penalty"] if sp.get("repetition_penalty") is not None else cfg.cb0_rep
    return {"frames": 0, "min": cfg.min_frames, "hazard": 0.0, "aeos": 0.0, "seed": s.seed, "ctr": 0, "hist": -1,
            "temp": sp.get("temperature") or cfg.cb0_temp, "top_k": sp.get("top_k") or cfg.cb0_top_k,
            "top_p": sp.get("top_p") or cfg.cb0_top_p, "rep": rep,
            "row_seed": (s.seed * 69069 + 1) % (2 ** 31 - 1), "row_ctr": 0, "lengths": 0}


def check_bind(eng, s):
    before = snapshot(eng)
    eng._bind(s)
    after = snapshot(eng)
    slot = s.slot
    for k, want in expected(eng, s).items():
        got = after[k][slot]
        # fp32 fields hold the request's value rounded once to fp32; integer fields are exact
        np.testing.assert_array_equal(got.numpy(), np.full(got.shape, want, dtype=got.numpy().dtype), err_msg=k)
    assert torch.equal(after["cross"][slot], eng.voice_const.cpu())
    for k in after:
        others = [i for i in range(after[k].shape[0]) if i != slot]
        assert torch.equal(after[k][others], before[k][others]), k


def test_bind_writes_every_field_of_the_slot_and_nothing_else(cuda):
    W = {k: v.to(cuda) for k, v in WG.generate(WG.all_shapes(TINY), seed=7).items()}
    eng = TickEngine(TINY, W, TickConfig(max_seats=3, capacity=64), device=cuda)
    rng = np.random.default_rng(0)
    dirty(eng)
    custom = eng.submit(rng.integers(0, TINY.backbone.vocab, 4), 10, sampling={
        "seed": 12345, "temperature": 0.55, "top_k": 7, "top_p": 0.85, "repetition_penalty": 1.25})
    eng.pending.remove(custom)
    check_bind(eng, custom)
    assert eng.cb0.any_top_p and eng.cb0.any_rep
    # a request with the engine's sampling after it, in the same slot
    eng._release(custom)
    dirty(eng)
    plain = eng.submit(rng.integers(0, TINY.backbone.vocab, 4), 10, seed=2 ** 31 - 2)
    eng.pending.remove(plain)
    check_bind(eng, plain)
    assert plain.slot == custom.slot
    # and a third request in another slot while the second holds its own
    other = eng.submit(rng.integers(0, TINY.backbone.vocab, 4), 10, sampling={"repetition_penalty": 0.0})
    eng.pending.remove(other)
    check_bind(eng, other)
    assert other.slot != plain.slot
    eng.close()


def test_slot_reset_rejects_bad_slots_and_misaligned_constants(cuda):
    W = {k: v.to(cuda) for k, v in WG.generate(WG.all_shapes(TINY), seed=7).items()}
    eng = TickEngine(TINY, W, TickConfig(max_seats=2, capacity=64), device=cuda)
    lib = L.load()
    src = eng.voice_const.data_ptr()

    def call(slot, cross):
        init = L.SlotInit(slot, 1, 2, 4, 8, 0, 0.9, 1.0, 0.8, cross)
        L.check(lib.m3_slot_reset(eng._slot_state, init, L.stream_ptr()), "m3_slot_reset")

    before = snapshot(eng)
    for slot in (-1, 2, 3, 1 << 20):          # the padding slot (max_slots) and beyond are not bindable
        with pytest.raises(IndexError, match="slot"):
            call(slot, src)
    with pytest.raises(ValueError, match="16-byte"):
        call(0, src + 2)                       # a speaker constant off its 16-byte boundary
    with pytest.raises(ValueError, match="null"):
        call(0, None)
    after = snapshot(eng)
    for k in after:
        assert torch.equal(after[k], before[k]), k
    call(1, src)
    after = snapshot(eng)
    assert after["seed"][1] == 1 and after["row_seed"][1] == 2 and after["min"][1] == 4 and after["top_k"][1] == 8
    assert eng.device_status() == 0
    eng.close()
