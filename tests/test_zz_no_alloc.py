"""m3_cb0_step_noalloc, the allocation-free cb0 step, against the regular m3_cb0_step.

Callers that cannot allocate device memory while they sample (a host that hands the library a fixed device budget
and forbids later cudaMalloc, or a latency-critical serving thread where cudaMalloc would synchronise the device)
use this entry point; its scratch is a static device array inside the library.  This file is collected last so that
a failure here cannot hide any other test's result; it passes alone in a fresh process and after the others.
"""
import ctypes

import numpy as np
import pytest
import torch

from conftest import golden
from maya2_native_b200 import _lib as L
from maya2_native_b200 import weights as WG
from maya2_native_b200.config import BASELINE, TINY
from maya2_native_b200.sampler import Cb0Sampler

pytestmark = pytest.mark.gpu
DEV_BAD_SLOT = 1


def _status(clear=True):
    """The allocation-free path's device status word (sticky across calls until read with clear=True)."""
    st = L.i32(-1)
    L.check(L.load().m3_cb0_noalloc_status(ctypes.byref(st), int(clear)), "m3_cb0_noalloc_status")
    return int(st.value)


def _noalloc(cfg, st, h, idx, rep, top_p):
    rows = int(idx.shape[0])
    code = torch.empty(rows, dtype=torch.long, device=h.device)
    cb0 = torch.empty(rows, dtype=torch.long, device=h.device)
    rc = L.load().m3_cb0_step_noalloc(ctypes.byref(cfg), ctypes.byref(st), h.data_ptr(), idx.data_ptr(),
                                      code.data_ptr(), cb0.data_ptr(), rows, rep, top_p, L.stream_ptr())
    L.check(rc, "m3_cb0_step_noalloc")
    torch.cuda.synchronize()
    return code, cb0


def _seed_state(s: Cb0Sampler, rng):
    m = s.max_slots + 1
    s.temp_t.copy_(torch.from_numpy(rng.uniform(0.5, 1.3, m).astype(np.float32)))
    s.topk_t.copy_(torch.from_numpy(rng.integers(1, 300, m)))
    s.topp_t[:] = 1.0
    s.topp_t[2] = 0.85
    s.rep_t.copy_(torch.from_numpy(rng.uniform(0, 2, m).astype(np.float32)))
    s.aeos_bias.copy_(torch.from_numpy(rng.uniform(0, 4, m).astype(np.float32)))
    s.seed_t.copy_(torch.from_numpy(rng.integers(1, 2 ** 31 - 1, m).astype(np.int32)))
    s.ctr_t.copy_(torch.from_numpy(rng.integers(0, 1000, m).astype(np.int32)))
    s.hist_t.copy_(torch.from_numpy(rng.integers(-1, 2048, s.hist_t.shape)))
    s.frames_t.copy_(torch.from_numpy(rng.integers(0, 40, m)))
    s.min_t[:] = 4
    s.hazard_t.copy_(torch.from_numpy(rng.uniform(0, 0.5, m).astype(np.float32)))
    s.any_top_p = True


def _state_struct(s: Cb0Sampler):
    return L.Cb0State(*[t.data_ptr() for t in (s.head, s.frames_t, s.min_t, s.hazard_t, s.aeos_bias, s.temp_t,
                                               s.topk_t, s.topp_t, s.rep_t, s.seed_t, s.ctr_t, s.hist_t)])


def test_noalloc_matches_cb0_step(cuda):
    _status()                                                # whatever an earlier call left: start from zero
    g = BASELINE.backbone
    head = WG.make("cb0_head.weight", (g.n_cb0, g.hidden))
    ref = Cb0Sampler(head, 12, max_rows=8, device=cuda)      # the regular, handle-based entry point
    own = Cb0Sampler(head, 12, max_rows=8, device=cuda)      # only its tensors are used: a second copy of the state
    for s in (ref, own):
        _seed_state(s, np.random.default_rng(7))
    lib = L.load()
    cfg = L.Cb0Config(g.hidden, g.n_cb0, 12, 8, own.rep_win)
    st = _state_struct(own)
    rng = np.random.default_rng(3)
    idx = torch.tensor([5, 0, 2, 11, 7], device=cuda)
    for call in range(2):           # two calls in a row: the shared scratch keeps the previous call's contents
        h = torch.from_numpy(rng.standard_normal((5, g.hidden)).astype(np.float32)).to(cuda, torch.bfloat16)
        code_r, cb0_r = ref(h, idx)
        code = torch.empty(5, dtype=torch.long, device=cuda)
        cb0 = torch.empty(5, dtype=torch.long, device=cuda)
        rep, top_p = own.flags()
        rc = lib.m3_cb0_step_noalloc(ctypes.byref(cfg), ctypes.byref(st), h.data_ptr(), idx.data_ptr(),
                                     code.data_ptr(), cb0.data_ptr(), 5, rep, top_p, L.stream_ptr())
        L.check(rc, "m3_cb0_step_noalloc")
        torch.cuda.synchronize()
        assert code.tolist() == code_r.tolist(), call
        assert cb0.tolist() == cb0_r.tolist(), call
        for name in ("ctr_t", "hist_t", "frames_t"):
            assert torch.equal(getattr(own, name), getattr(ref, name)), (call, name)
        torch.testing.assert_close(own.hazard_t, ref.hazard_t, rtol=1e-6, atol=1e-7)
    # the row limit itself: 8 rows in one call
    idx = torch.tensor([1, 3, 4, 6, 8, 9, 10, 11], device=cuda)
    h = torch.from_numpy(rng.standard_normal((8, g.hidden)).astype(np.float32)).to(cuda, torch.bfloat16)
    code_r, cb0_r = ref(h, idx)
    rep, top_p = own.flags()
    code, cb0 = _noalloc(cfg, st, h, idx, rep, top_p)
    assert code.tolist() == code_r.tolist() and cb0.tolist() == cb0_r.tolist()
    assert torch.equal(own.hist_t, ref.hist_t)
    assert _status() == 0


def test_noalloc_matches_reference_fixture(cuda):
    """Pinned to the reference's own Engine._cb0 on the same hidden states (tests/golden/cb0_sampler.npz): stop codes
    exact; the bf16 head GEMM may differ from the reference's by an ulp, so one sampled code may move (the same bar
    as the handle-based entry point's test)."""
    _status()
    g = TINY.backbone
    z = golden("cb0_sampler.npz")
    s = Cb0Sampler(WG.make("cb0_head.weight", (g.n_cb0, g.hidden)), 5, max_rows=8, device=cuda)
    for name in ("temp_t", "topk_t", "topp_t", "rep_t", "aeos_bias", "seed_t", "ctr_t", "hist_t", "frames_t",
                 "min_t", "hazard_t"):
        getattr(s, name).copy_(torch.from_numpy(z["init_" + name]))
    cfg = L.Cb0Config(g.hidden, g.n_cb0, 5, 8, s.rep_win)
    st = _state_struct(s)
    idx = torch.arange(5, device=cuda)
    miss = 0
    for it in range(3):
        h = torch.from_numpy(z[f"h{it}"]).to(cuda, torch.bfloat16)
        code, cb0 = _noalloc(cfg, st, h, idx, 1, 1)          # the fixture's engine had a penalty and top-p request
        assert code.cpu().tolist() == z[f"code{it}"].tolist(), it
        miss += int((cb0.cpu().numpy() != z[f"cb0{it}"]).sum())
    assert miss <= 1
    assert s.ctr_t.cpu().tolist() == z["final_ctr_t"].tolist()
    assert s.frames_t.cpu().tolist() == z["final_frames_t"].tolist()
    assert _status() == 0


def test_noalloc_reports_a_bad_slot(cuda):
    """A slot outside [0, max_slots] (which the host-side mirror would reject) is sampled from the padding slot's
    state, the other rows are unaffected, and the status word says so until it is read and cleared."""
    _status()
    g = BASELINE.backbone
    head = WG.make("cb0_head.weight", (g.n_cb0, g.hidden))
    ref = Cb0Sampler(head, 12, max_rows=8, device=cuda)
    own = Cb0Sampler(head, 12, max_rows=8, device=cuda)
    for s in (ref, own):
        _seed_state(s, np.random.default_rng(11))
    cfg = L.Cb0Config(g.hidden, g.n_cb0, 12, 8, own.rep_win)
    st = _state_struct(own)
    h = torch.from_numpy(np.random.default_rng(5).standard_normal((2, g.hidden)).astype(np.float32)).to(
        cuda, torch.bfloat16)
    code_r, cb0_r = ref(h, torch.tensor([4, 12], device=cuda))       # slot 12 = the padding slot
    rep, top_p = own.flags()
    code, cb0 = _noalloc(cfg, st, h, torch.tensor([4, 99], device=cuda), rep, top_p)
    assert code.tolist() == code_r.tolist() and cb0.tolist() == cb0_r.tolist()
    assert _status(clear=False) == DEV_BAD_SLOT
    code, cb0 = _noalloc(cfg, st, h[:1], torch.tensor([5], device=cuda), rep, top_p)   # a good call keeps it
    assert _status() == DEV_BAD_SLOT                          # read and clear
    assert _status() == 0


def test_noalloc_rejects_oversized_calls(cuda):
    g = BASELINE.backbone
    s = Cb0Sampler(WG.make("cb0_head.weight", (g.n_cb0, g.hidden)), 12, max_rows=16, device=cuda)
    cfg = L.Cb0Config(g.hidden, g.n_cb0, 12, 16, s.rep_win)
    st = _state_struct(s)
    h = torch.zeros(9, g.hidden, dtype=torch.bfloat16, device=cuda)
    idx = torch.zeros(9, dtype=torch.long, device=cuda)
    out = torch.empty(9, dtype=torch.long, device=cuda)
    rc = L.load().m3_cb0_step_noalloc(ctypes.byref(cfg), ctypes.byref(st), h.data_ptr(), idx.data_ptr(),
                                      out.data_ptr(), out.data_ptr(), 9, 1, 0, L.stream_ptr())
    assert rc == L.M3_ERR_ARG
    assert b"rows" in L.load().m3_last_error()
    # a hidden-state pointer off a 16-byte boundary is refused before any device work
    hb = torch.zeros(2 * g.hidden + 8, dtype=torch.bfloat16, device=cuda)
    rc = L.load().m3_cb0_step_noalloc(ctypes.byref(cfg), ctypes.byref(st), hb.data_ptr() + 2, idx.data_ptr(),
                                      out.data_ptr(), out.data_ptr(), 2, 1, 0, L.stream_ptr())
    assert rc == L.M3_ERR_ARG
    assert b"16-byte" in L.load().m3_last_error()
