"""GPU parity of the one-frame streaming Mimi decoder (m3_mimi_decode via the StaticMimi mirror): PCM SNR above
30 dB against the reference's own StaticMimi (fixture, with slot resets and a wrapped KV ring) and against the bf16
oracle at the benchmark geometry over more frames than the 256-entry ring holds."""
import numpy as np
import pytest
import torch

from conftest import golden
from maya2_native_b200 import weights as WG
from maya2_native_b200.codec import StaticMimi
from maya2_native_b200.config import BASELINE, TINY
from oracle.mimi import MimiOracle

pytestmark = pytest.mark.gpu


def snr_db(x, ref):
    x, ref = np.asarray(x, np.float64), np.asarray(ref, np.float64)
    return 10 * np.log10(np.sum(ref ** 2) / max(np.sum((x - ref) ** 2), 1e-30))


def test_tiny_matches_reference_fixture(cuda):
    g = TINY.mimi
    z = golden("mimi_tiny_bf16.npz")
    sm = StaticMimi(WG.mimi_weights(g), 3, batch_buckets=(1, 2, 4), ring=g.ring, geom=g, device=cuda)
    got, ref = [], []
    for f in range(24):
        if f == 5:
            sm.reset(2)
        if f == 14:
            sm.reset(1)
        slots = z[f"slots{f}"].tolist()
        pcm = sm.decode(slots, torch.from_numpy(z[f"codes{f}"]).to(cuda))
        got.append(pcm.cpu().numpy())
        ref.append(z[f"pcm{f}"])
    assert snr_db(np.concatenate(got), np.concatenate(ref)) > 30
    assert sm.device_status() == 0


def test_baseline_geometry_wraps_ring_against_oracle(cuda):
    g = BASELINE.mimi
    W = WG.mimi_weights(g)
    B = 3
    sm = StaticMimi(W, B, batch_buckets=(B,), geom=g, device=cuda)
    orc = MimiOracle({k: v.numpy() for k, v in W.items()}, g, B, "bf16")
    rng = np.random.default_rng(0)
    got, ref = [], []
    for f in range(132):          # 264 transformer tokens > the 256-entry ring
        if f == 40:
            sm.reset(1)
            orc.reset(1)
        codes = rng.integers(0, g.codebook_size, (B, g.n_q))
        slots = [0, 1, 2] if f % 2 else [2, 0, 1]
        got.append(sm.decode(slots, torch.from_numpy(codes).to(cuda)).cpu().numpy())
        ref.append(orc.decode(np.array(slots), codes))
    snr = snr_db(np.concatenate(got), np.concatenate(ref))
    assert snr > 30, snr
    assert sm.tokens[:B].cpu().tolist() == orc.tokens[:B].tolist()
    assert sm.device_status() == 0


def test_many_streams_against_oracle_subset(cuda):
    """160 streams, so the persistent SEANet kernels walk several tiles per CTA (buffer alternation, the next tile's
    load overlapping the current one); streams are independent, so the oracle decodes a subset of them (first,
    middle and last slots) from the same codes over three frames (the stage histories and tails cross frames)."""
    g = BASELINE.mimi
    W = WG.mimi_weights(g)
    B = 160
    pick = [0, 1, 79, 158, 159]
    sm = StaticMimi(W, B, batch_buckets=(B,), geom=g, device=cuda)
    orc = MimiOracle({k: v.numpy() for k, v in W.items()}, g, len(pick), "bf16")
    rng = np.random.default_rng(3)
    for f in range(3):
        codes = rng.integers(0, g.codebook_size, (B, g.n_q))
        got = sm.decode(list(range(B)), torch.from_numpy(codes).to(cuda)).cpu().numpy()
        ref = orc.decode(np.arange(len(pick)), codes[pick])
        for i, s in enumerate(pick):
            assert snr_db(got[s], ref[i]) > 30, (f, s, snr_db(got[s], ref[i]))
    assert sm.device_status() == 0


def test_sm_budget_changes_no_result(cuda):
    """The SEANet kernels spread over a few SMs (the engine's codec beside the next tick) give the same PCM, bit for
    bit, as over all of them: the budget sets the grid of the persistent kernels, not their arithmetic."""
    g = BASELINE.mimi
    B = 48
    W = WG.generate(WG.mimi_shapes(g), seed=4, device=cuda)
    pcm = {}
    for sms in (0, 9):
        sm = StaticMimi(W, B, batch_buckets=(B,), geom=g, device=cuda)
        sm.set_sm_budget(sms)
        gen = torch.Generator(device=cuda).manual_seed(9)
        idx = torch.arange(B, device=cuda)
        out = []
        for _ in range(4):
            codes = torch.randint(0, g.codebook_size, (B, g.n_q), device=cuda, generator=gen)
            out.append(sm.decode(idx, codes).cpu())
        assert sm.device_status() == 0
        pcm[sms] = torch.cat(out)
        sm.close()
    assert torch.equal(pcm[0], pcm[9])
