"""GPU parity of the depth level loop (m3_depth_step via the FastDepth mirror) against the reference's fixtures
(its fused bf16 body with Philox sampling) and the bf16 oracle at the benchmark geometry."""
import numpy as np
import pytest
import torch

from conftest import golden
from maya2_native_b200 import weights as WG
from maya2_native_b200.config import BASELINE, TINY, DepthGeom
from maya2_native_b200.depth import FastDepth
from oracle.depth import DepthOracle

pytestmark = pytest.mark.gpu


def rel_l2(a, b):
    a, b = np.asarray(a, np.float32), np.asarray(b, np.float32)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))


def _fd(W, g, cuda, greedy, B=3, **kw):
    fd = FastDepth(W, B, temp=0.8, top_k=50, batch_buckets=(B,), seed=7, greedy=greedy, geom=g, device=cuda, **kw)
    return fd


@pytest.mark.parametrize("greedy", [True, False])
def test_tiny_matches_reference_fixture(cuda, greedy):
    g = TINY.depth
    z = golden("depth_tiny_bf16.npz")
    fd = _fd(WG.depth_weights(g), g, cuda, greedy)
    for s in range(3):
        fd.set_speaker(s, torch.from_numpy(z["mems"][s]), torch.ones(1, 1, dtype=torch.bool))
    fd.row_seed[:3] = torch.tensor([11, 22, 2 ** 31 - 3], dtype=torch.int32)
    tag = "g" if greedy else "s"
    slots = z["slots"].tolist()
    agree, total = 0, 0
    for f in range(2):
        h = torch.from_numpy(z[f"{tag}_h{f}"]).to(cuda, torch.bfloat16)
        cb0 = torch.from_numpy(z[f"{tag}_cb0_{f}"]).to(cuda)
        codes, fb = fd(slots, h, cb0)
        ref = z[f"{tag}_codes{f}"]
        agree += int((codes.cpu().numpy() == ref).sum())
        total += ref.size
        if (codes.cpu().numpy() == ref).all():
            assert rel_l2(fb.float().cpu(), z[f"{tag}_fb{f}"]) < 2e-2
    # greedy is decided by argmax of nearly identical logits; sampled codes additionally ride the same Philox noise
    assert agree / total >= (1.0 if greedy else 0.9)
    assert fd.row_ctr[:3].cpu().tolist() == z[f"{tag}_row_ctr"][:3].tolist()
    assert fd.device_status() == 0


def _oracle_vs_gpu(g, cuda, B, frames, greedy, seed=0, forced=False):
    W = WG.depth_weights(g)
    fd = FastDepth(W, B, temp=0.8, top_k=50, batch_buckets=(B,), seed=7, greedy=greedy, geom=g, device=cuda)
    orc = DepthOracle({k: v.numpy() for k, v in W.items()}, g, B, "bf16", temp=0.8, top_k=50, greedy=greedy)
    rng = np.random.default_rng(seed)
    for s in range(B):
        mem = rng.standard_normal(g.d).astype(np.float32)
        fd.set_speaker(s, torch.from_numpy(mem).view(1, 1, -1), torch.ones(1, 1, dtype=torch.bool))
        orc.set_speaker(s, torch.from_numpy(mem).to(torch.bfloat16).float().numpy(), 1.0)
    seeds = rng.integers(1, 2 ** 31 - 1, B)
    fd.row_seed[:B] = torch.from_numpy(seeds).to(torch.int32)
    orc.row_seed[:B] = seeds
    slots = list(range(B))[::-1]
    agree, total, fb_err, gaps = 0, 0, [], []
    for f in range(frames):
        h = torch.from_numpy(rng.standard_normal((B, g.d_backbone)).astype(np.float32)).to(torch.bfloat16)
        cb0 = rng.integers(0, g.n_codes, B)
        codes, fb = fd(slots, h.to(cuda), torch.from_numpy(cb0).to(cuda))
        gc = codes.cpu().numpy()
        # forced: the oracle's prefix follows the GPU's codes, so every level is compared from the same inputs and
        # one flipped near-tie does not change the levels after it
        rc, rfb = orc.step(slots, h.float().numpy(), cb0, force=gc if forced else None)
        c0 = 1 if forced else 0  # forced: count the sampled levels only (column 0 is the given cb0)
        agree += int((gc[:, c0:] == rc[:, c0:]).sum())
        total += rc[:, c0:].size
        if forced and greedy:  # how far apart, in the oracle's own logits, are the two picks of a flipped decision
            for lv in range(1, rc.shape[1]):
                for r in np.nonzero(gc[:, lv] != rc[:, lv])[0]:
                    lg = np.asarray(orc.last_logits[lv - 1][r], np.float64)
                    gaps.append((lg[rc[r, lv]] - lg[gc[r, lv]]) / max(abs(lg[rc[r, lv]]), 1e-30))
        same = (codes.cpu().numpy() == rc).all(1)
        if same.any():
            fb_err.append(rel_l2(fb.float().cpu().numpy()[same], rfb[same]))
    assert fd.device_status() == 0
    if forced and greedy:
        return agree / total, max(fb_err) if fb_err else 0.0, max(gaps) if gaps else 0.0
    return agree / total, max(fb_err) if fb_err else 0.0


def test_grouped_levels_incremental_path(cuda):
    """Shared band groups (levels 9-11 share one trunk) exercise the incremental K/V path."""
    g = DepthGeom(layers=2, d=128, heads=2, ffn=256, n_q=12, rank=16, d_backbone=256)
    acc, err = _oracle_vs_gpu(g, cuda, B=6, frames=3, greedy=True)
    assert acc >= 0.97 and err < 2e-2


@pytest.mark.parametrize("greedy", [True, False])
def test_baseline_geometry_against_oracle(cuda, greedy):
    """8 seats x 25 frames x 7 levels at the benchmark geometry, each level from the GPU's own prefix (a flip at one
    level does not carry into the next), greedy and sampled (per-seat Philox streams): at least 98% of the decisions
    agree with the bf16-emulating oracle, as over 200 frames below; greedy flips are near ties in the oracle's own
    logits."""
    res = _oracle_vs_gpu(BASELINE.depth, cuda, B=8, frames=25, greedy=greedy, seed=11, forced=True)
    acc, err = res[0], res[1]
    print(f"benchmark-geometry depth agreement ({'greedy' if greedy else 'sampled'}): {acc:.4f}")
    assert acc >= 0.98 and err < 2e-2, (acc, err)
    if greedy:
        assert res[2] <= 2.0 ** -6, res[2]


def test_baseline_geometry_greedy_agreement_over_200_frames(cuda):
    """Greedy code agreement over 200 frames (2 seats x 7 levels): the GPU's bf16 level loop against the
    bf16-emulating oracle, every frame from the same hidden state and cb0, each level from the GPU's own prefix.  The
    logits are bf16 values in the reference too (its heads are bf16 linears), so two correct implementations that
    accumulate in different orders disagree where the top two logits are within a rounding step: with random-init
    weights that is about 1.4% of the decisions (98.6% agreement measured), and every disagreement must be such a
    near tie in the oracle's own logits."""
    acc, err, gap = _oracle_vs_gpu(BASELINE.depth, cuda, B=2, frames=200, greedy=True, seed=5, forced=True)
    print("greedy agreement over 200 frames (teacher-forced levels):", acc, "largest flipped gap:", gap)
    assert acc >= 0.98 and err < 2e-2, (acc, err)
    assert gap <= 2.0 ** -6, gap          # within a few bf16 steps of each other
