"""Failure detection on the GPU without a fault: every kernel of the library checks the indices it is handed and
every wait it makes is bounded; what goes wrong is recorded in the handle's device status word, which the host
reads after the step (the reference raises on the host; a C caller that skips the host checks still gets a
contained, reported error).  The failures are made on the host side -- an index the host checks would have
rejected, a barrier nothing arrives on -- so no access leaves its buffer and the context stays usable."""
import ctypes

import pytest
import torch

from maya2_native_b200 import _lib as L
from maya2_native_b200 import weights as WG
from maya2_native_b200.backbone import StaticBackbone
from maya2_native_b200.config import TINY
from maya2_native_b200.sampler import Cb0Sampler

pytestmark = pytest.mark.gpu
DEV_BAD_SLOT, DEV_BAD_POS, DEV_TIMEOUT = 1, 2, 4


def test_bounded_wait_gives_up_and_reports(cuda):
    st = L.i32(-1)
    L.check(L.load().m3_selftest_timeout(1000, ctypes.byref(st)), "m3_selftest_timeout")
    assert st.value == DEV_TIMEOUT, L.DEV_STATUS.get(st.value)
    x = torch.arange(8, device=cuda, dtype=torch.float32)       # the context is still healthy
    assert float(x.sum()) == 28.0


def test_attention_waits_run_out_and_report(cuda):
    """The decode attention's own bounded waits (m3_backbone_attention_selftest: every K/V stage barrier expects 16
    bytes more than its copies bring, so every wait runs out): the launch ends by itself, the handle's status reads
    M3_DEV_TIMEOUT, and the same context then steps exactly as a backbone that never timed out."""
    g = TINY.backbone
    W = WG.backbone_weights(g)
    mk = lambda: StaticBackbone(W, 2, capacity=64, ctx_buckets=(64,), batch_buckets=(1, 2), use_graphs=False, geom=g,
                                device=cuda)
    a, b = mk(), mk()
    x1 = torch.randn(2, g.hidden, device=cuda, dtype=torch.bfloat16)
    x2 = torch.randn(2, g.hidden, device=cuda, dtype=torch.bfloat16)
    for sb in (a, b):
        sb.step([0, 1], x1)
    L.check(L.load().m3_backbone_attention_selftest(a._handle, 0, 2, 64, L.stream_ptr()),
            "m3_backbone_attention_selftest")
    torch.cuda.synchronize()
    assert a.device_status() == DEV_TIMEOUT
    assert a.device_status() == 0                       # read and cleared
    ya, yb = a.step([0, 1], x2), b.step([0, 1], x2)
    assert torch.equal(ya, yb)
    assert a.device_status() == 0 and b.device_status() == 0


def _raw_step(sb, slots, x, ctx):
    """m3_backbone_step through the C ABI, without the mirror's host-side slot validation."""
    rows = len(slots)
    s = torch.tensor(slots, device=x.device, dtype=torch.int64)
    off = torch.zeros(rows, device=x.device, dtype=torch.int64)
    real = torch.ones(rows, device=x.device, dtype=torch.int64)
    out = torch.empty_like(x)
    rc = L.load().m3_backbone_step(sb._handle, s.data_ptr(), off.data_ptr(), real.data_ptr(), x.data_ptr(),
                                   out.data_ptr(), rows, ctx, L.stream_ptr())
    torch.cuda.synchronize()
    return rc, out


def test_bad_slot_and_position_are_contained_and_reported(cuda):
    g = TINY.backbone
    sb = StaticBackbone(WG.backbone_weights(g), 3, capacity=64, ctx_buckets=(64,), batch_buckets=(4,), geom=g,
                        device=cuda)
    x = torch.randn(2, g.hidden, device=cuda).to(torch.bfloat16)
    rc, ref = _raw_step(sb, [0, 1], x, 64)
    assert rc == 0 and sb.device_status() == 0
    with torch.inference_mode():                                # the mirror's lengths are inference tensors
        sb.lengths[:3] = 0
    # a slot past max_slots: the row is redirected to the padding slot, the other row is untouched
    rc, out = _raw_step(sb, [0, 99], x, 64)
    assert rc == 0
    assert sb.device_status() == DEV_BAD_SLOT
    assert sb.device_status() == 0                              # read-and-clear
    assert torch.isfinite(out.float()).all()
    assert torch.equal(out[0], ref[0])
    # a slot whose KV is full: the position is clamped to the last entry and reported
    with torch.inference_mode():
        sb.lengths[1] = 64
    rc, out = _raw_step(sb, [1], x[:1], 64)
    assert rc == 0
    assert sb.device_status() == DEV_BAD_POS
    assert torch.isfinite(out.float()).all()
    sb.close()


def test_cb0_bad_slot_is_contained_and_reported(cuda):
    """The cb0 handle: a row naming a slot past max_slots is sampled from the padding slot's state and reported in
    the handle's status word; both rows equal a clean call that names the padding slot itself."""
    g = TINY.backbone
    head = WG.make("cb0_head.weight", (g.n_cb0, g.hidden))
    ref = Cb0Sampler(head, 3, max_rows=4, device=cuda)
    s = Cb0Sampler(head, 3, max_rows=4, device=cuda)
    for x in (ref, s):
        x.seed_t[:] = 7
    h = torch.randn(2, g.hidden, device=cuda).to(torch.bfloat16)
    code_r, cb0_r = ref(h, torch.tensor([1, 3], device=cuda))           # slot 3 = the padding slot
    code, cb0 = s(h, torch.tensor([1, 99], device=cuda))
    torch.cuda.synchronize()
    assert s.device_status() == DEV_BAD_SLOT
    assert s.device_status() == 0                               # read-and-clear
    assert ref.device_status() == 0
    assert code.tolist() == code_r.tolist() and cb0.tolist() == cb0_r.tolist()
    s.close()
    ref.close()
