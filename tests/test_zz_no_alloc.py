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

from maya2_native_b200 import _lib as L
from maya2_native_b200 import weights as WG
from maya2_native_b200.config import BASELINE
from maya2_native_b200.sampler import Cb0Sampler

pytestmark = pytest.mark.gpu


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
