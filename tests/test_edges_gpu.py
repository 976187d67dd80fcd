"""Edge cases on the GPU, as the reference's serve objects treat them: empty calls, zero-row C ABI calls, and the
largest calls each object allows -- a full row bucket whose prefill ends exactly at the KV capacity, the last slot
before the padding slot, and the extreme code values -- checked against the oracle."""
import numpy as np
import pytest
import torch

from maya2_native_b200 import _lib as L
from maya2_native_b200 import weights as WG
from maya2_native_b200.backbone import StaticBackbone
from maya2_native_b200.codec import StaticMimi
from maya2_native_b200.config import TINY
from maya2_native_b200.depth import FastDepth
from oracle.backbone import BackboneOracle
from oracle.depth import DepthOracle
from oracle.mimi import MimiOracle

pytestmark = pytest.mark.gpu


def rel_maxabs(a, b):
    a, b = np.asarray(a, np.float32), np.asarray(b, np.float32)
    return float(np.abs(a - b).max() / max(1.0, np.abs(b).max()))


def test_backbone_empty_and_full_bucket_at_capacity(cuda):
    """step([]) returns an empty batch (serve/fast_backbone.py:291); a zero-row C ABI step is a no-op; then one step
    of exactly the largest row bucket (3 decode rows + a 5-row inline prefill) on the last real slot, whose prefill
    fills the KV cache to the last position -- against the oracle, and one more row is refused."""
    g = TINY.backbone
    W = WG.backbone_weights(g)
    cap, slots = 32, 4
    sb = StaticBackbone(W, slots, capacity=cap, ctx_buckets=(cap,), batch_buckets=(1, 8), geom=g, device=cuda)
    orc = BackboneOracle({k: v.numpy() for k, v in W.items()}, g, slots, cap, "bf16")
    x0 = torch.zeros(0, g.hidden, device=cuda, dtype=torch.bfloat16)
    assert tuple(sb.step([], x0).shape) == (0, g.hidden)
    z = torch.zeros(8, dtype=torch.long, device=cuda)
    xz = torch.zeros(8, g.hidden, device=cuda, dtype=torch.bfloat16)
    rc = L.load().m3_backbone_step(sb._handle, z.data_ptr(), z.data_ptr(), z.data_ptr(), xz.data_ptr(),
                                   xz.data_ptr(), 0, cap, L.stream_ptr())
    assert rc == L.M3_OK
    rng = np.random.default_rng(3)
    # slots 0..2 hold 8 positions; slot 3 (the last real slot) holds 27 so that 5 prefill rows reach position 31;
    # prefills go in chunks of the largest row bucket (8)
    pre = {0: 8, 1: 8, 2: 8, 3: cap - 5}
    for s, n in pre.items():
        x = rng.standard_normal((n, g.hidden)).astype(np.float32)
        for c0 in range(0, n, 8):
            xc = torch.from_numpy(x[c0:c0 + 8]).to(torch.bfloat16)
            _, last = sb.step_mixed([], None, [(s, xc.to(cuda))])
            _, olast = orc.step_mixed([], None, [(s, xc.float().numpy())])
            assert rel_maxabs(last[0].float().cpu(), olast[0]) < 2e-2
    xd = rng.standard_normal((3, g.hidden)).astype(np.float32)
    xp = rng.standard_normal((5, g.hidden)).astype(np.float32)
    bf = lambda a: torch.from_numpy(a).to(torch.bfloat16)
    dec, last = sb.step_mixed([0, 1, 2], bf(xd).to(cuda), [(3, bf(xp).to(cuda))])
    odec, olast = orc.step_mixed([0, 1, 2], bf(xd).float().numpy(), [(3, bf(xp).float().numpy())])
    assert rel_maxabs(dec.float().cpu(), odec) < 2e-2
    assert rel_maxabs(last[0].float().cpu(), olast[0]) < 2e-2
    assert sb.lengths_cpu[3] == cap and int(sb.lengths[3]) == cap
    with pytest.raises(ValueError):
        sb.step([3], bf(xd[:1]).to(cuda))        # the KV cache of slot 3 is full
    with pytest.raises(IndexError):
        sb.step([slots], bf(xd[:1]).to(cuda))    # slot max_slots is the padding slot
    assert sb.device_status() == 0


def test_depth_empty_and_extreme_codes(cuda):
    """FastDepth with no seats returns empty codes and feedback (serve/fast_depth.py:241-257 runs its smallest
    bucket); a full bucket with the last real slot and cb0 at 0 and 2047 matches the greedy oracle."""
    g = TINY.depth
    W = WG.depth_weights(g)
    B = 4
    fd = FastDepth(W, B, batch_buckets=(1, B), greedy=True, geom=g, device=cuda)
    orc = DepthOracle({k: v.numpy() for k, v in W.items()}, g, B, "bf16", greedy=True)
    null = W["depth.null_mem"].reshape(1, 1, -1)
    for s in range(B):
        fd.set_speaker(s, null, torch.ones(1, 1, dtype=torch.bool))
        orc.set_speaker(s, null.reshape(-1).to(torch.bfloat16).float().numpy(), 1.0)
    codes, fb = fd([], torch.zeros(0, g.d_backbone, device=cuda, dtype=torch.bfloat16),
                   torch.zeros(0, dtype=torch.long, device=cuda))
    assert tuple(codes.shape) == (0, g.n_q) and tuple(fb.shape) == (0, g.d_backbone)
    h = torch.from_numpy(np.random.default_rng(4).standard_normal((B, g.d_backbone)).astype(np.float32))
    h = h.to(torch.bfloat16)
    cb0 = np.array([0, g.n_codes - 1, 5, g.n_codes - 1])
    slots = [3, 0, 2, 1]
    codes, fb = fd(slots, h.to(cuda), torch.from_numpy(cb0).to(cuda))
    ocodes, ofb = orc.step(slots, h.float().numpy(), cb0, force=codes.cpu().numpy())
    got = codes.cpu().numpy()
    assert (got[:, 0] == cb0).all() and (got >= 0).all() and (got < g.n_codes).all()
    assert (got == ocodes).mean() >= 0.9
    assert rel_maxabs(fb.float().cpu(), ofb) < 2e-2
    assert fd.device_status() == 0


def test_mimi_empty_and_extreme_codes(cuda):
    """StaticMimi.decode of no slots raises ValueError as the reference's does (serve/fast_codec.py:258: min() of an
    empty list); a zero-row C ABI decode is a no-op; a full bucket with the last real slot and codes 0 / 2047
    matches the oracle."""
    g = TINY.mimi
    W = WG.mimi_weights(g)
    B = 4
    sm = StaticMimi(W, B, batch_buckets=(B,), ring=g.ring, geom=g, device=cuda)
    orc = MimiOracle({k: v.numpy() for k, v in W.items()}, g, B, "bf16")
    with pytest.raises(ValueError):
        sm.decode([], torch.zeros(0, g.n_q, dtype=torch.long, device=cuda))
    z = torch.zeros(1, dtype=torch.long, device=cuda)
    assert L.load().m3_mimi_decode(sm._handle, z.data_ptr(), z.data_ptr(), z.data_ptr(), 0, L.stream_ptr()) == L.M3_OK
    slots = [3, 1, 0, 2]
    got, ref = [], []
    for f in range(3):
        codes = np.zeros((B, g.n_q), np.int64)
        codes[1] = g.codebook_size - 1
        codes[2, ::2] = g.codebook_size - 1
        codes[3] = np.random.default_rng(f).integers(0, g.codebook_size, g.n_q)
        got.append(sm.decode(slots, torch.from_numpy(codes).to(cuda)).cpu().numpy())
        ref.append(orc.decode(np.array(slots), codes))
    got, ref = np.concatenate(got), np.concatenate(ref)
    snr = 10 * np.log10((ref ** 2).sum() / max(((got - ref) ** 2).sum(), 1e-30))
    assert snr > 30, snr
    assert sm.device_status() == 0


def test_single_call_tick_equals_the_two_stream_tick(cuda):
    """m3_tick_run (main part, codec hand-off and codec part in order on one stream: the C ABI's one-call tick)
    delivers the same packed readout, bit for bit, as TickEngine's tick with the codec part on its own stream beside
    the next tick's main part, tick by tick over admissions and decode ticks."""
    from maya2_native_b200.engine import TickConfig, TickEngine
    W = {k: v.to(cuda) for k, v in WG.generate(WG.all_shapes(TINY), seed=12).items()}
    cfg = TickConfig(max_seats=3, capacity=64, max_inline_rows=8, stops=False)
    rng = np.random.default_rng(12)
    prompts = [rng.integers(0, TINY.backbone.vocab, n) for n in (5, 3, 4, 6)]
    engines = [TickEngine(TINY, W, cfg, device=cuda) for _ in range(2)]
    for e in engines:
        for i, p in enumerate(prompts):
            e.submit(p, 6 + i, seed=40 + i)
    lib = L.load()
    two, one = engines
    for _ in range(12):
        out = two.tick_pipelined()
        got_two = two.last_readout().copy() if out else None
        # the same tick through the one-call entry point on the other engine
        new = one._admit()
        dec = list(one.active)
        if not dec and not new:
            break
        tp = one.make_plan(dec, new)
        plan = torch.from_numpy(tp.plan).to(cuda)
        packed = torch.zeros(tp.seats, 2 + one.spf // 4, dtype=torch.long, device=cuda)
        rep, top_p = one.cb0.flags()
        torch.cuda.current_stream().wait_stream(one.codec_stream)   # the admitted slots' codec resets
        assert lib.m3_tick_run(one._handle, plan.data_ptr(), tp.rows, tp.seats, tp.ctx, rep, top_p,
                               packed.data_ptr(), L.stream_ptr()) == L.M3_OK
        one.commit(tp)
        hv = packed[:len(dec) + len(new)].cpu().numpy()
        one._deliver(tp.dec + tp.new, hv)
        if got_two is not None:
            assert np.array_equal(got_two, ref_prev), "readout of the previous tick differs"
        ref_prev = hv
    for s in two.flush():
        pass
    assert np.array_equal(two.last_readout(), ref_prev)
    assert two.device_status() == 0 and one.device_status() == 0
    for e in engines:
        e.close()
