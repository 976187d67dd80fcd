"""Pin the CPU oracle to the reference: every fixture in tests/golden was produced by running the reference's own
code (tests/golden/make_golden.py) on the same seeded weights.  CPU only."""
import numpy as np
import pytest

from conftest import golden
from maya2_native_b200 import weights as WG
from maya2_native_b200.config import TINY, DepthGeom
from oracle.backbone import BackboneOracle
from oracle.depth import DepthOracle
from oracle.mimi import MimiOracle
from oracle.philox import uniform
from oracle.sampler import Cb0State, cb0_sample, row_exponential, topk_sample


@pytest.fixture(scope="module")
def bb_weights():
    return {k: v.numpy() for k, v in WG.backbone_weights(TINY.backbone).items()}


@pytest.mark.parametrize("dtype,tol", [("fp32", 1e-5), ("bf16", 1e-2)])
def test_backbone(bb_weights, dtype, tol):
    """fp32: the reference's gather path to ~1e-6.  bf16: its fused Triton path (interpreted, RNE casts) bit-for-bit
    except for rare 1-ulp accumulation-order differences."""
    z = golden(f"backbone_tiny_{dtype}.npz")
    o = BackboneOracle(bb_weights, TINY.backbone, 3, 64, dtype)
    exact = 0
    for i in range(6):
        y = o.forward(z[f"slots{i}"], z[f"x{i}"], z[f"offsets{i}"])
        ref = z[f"out{i}"]
        assert np.abs(y - ref).max() <= tol * max(1.0, np.abs(ref).max())
        exact += int((y == ref).all())
    assert o.lengths.tolist() == z["lengths"].tolist()
    assert np.abs(o.k[-1][:3, :, :12] - z["k_last"]).max() <= tol * 4
    if dtype == "bf16":
        assert exact >= 4          # most steps identical to the last bit


def test_philox_matches_tl_rand_stream():
    """row_exponential's first entries for known (seed, counter) pairs, printed by the reference kernel."""
    e = row_exponential(np.array([5, 6, 7]), np.array([0, 1, 2]), 4, 0)
    np.testing.assert_allclose(e, [[0.75921077, 0.36464632, 2.6226392, 0.41574517],
                                   [0.60396683, 0.8941197, 1.1294045, 0.89487416],
                                   [1.2329998, 0.3962875, 1.230995, 2.6444952]], rtol=1e-6)
    u = uniform(np.array([1, 2 ** 31 - 1]), np.array([0, 123456789]))
    assert ((u >= 0) & (u < 1)).all()


def test_topk_sampler_bit_exact():
    z = golden("topk_sampler.npz")
    for level in (1, 5, 31):
        for k in (1, 50, 64, 2048):
            got = topk_sample(z["logits"], z["seeds"], z["ctrs"], level, 0.7, k)
            assert (got == z[f"s_l{level}_k{k}"]).all()
        assert (topk_sample(z["logits"], z["seeds"], z["ctrs"], level, 0.8, 50, True) == z[f"g_l{level}"]).all()
    assert (topk_sample(z["logits_bf16"], z["seeds"], z["ctrs"], 3, 0.8, 50) == z["s_bf16"]).all()


def test_cb0_sampler_bit_exact(bb_weights):
    z = golden("cb0_sampler.npz")
    st = Cb0State(5)
    for a, b in {"temp": "temp_t", "topk": "topk_t", "topp": "topp_t", "rep": "rep_t", "aeos_bias": "aeos_bias",
                 "seed": "seed_t", "ctr": "ctr_t", "hist": "hist_t", "frames": "frames_t", "min": "min_t",
                 "hazard": "hazard_t"}.items():
        setattr(st, a, z["init_" + b].astype(getattr(st, a).dtype))
    o = BackboneOracle(bb_weights, TINY.backbone, 3, 64, "bf16")
    for it in range(3):
        assert np.abs(o.cb0_logits(z[f"h{it}"]) - z[f"logits{it}"]).max() <= 2 ** -6
        code, cb0 = cb0_sample(z[f"logits{it}"], np.arange(5), st, True, True)
        assert code.tolist() == z[f"code{it}"].tolist()
        assert cb0.tolist() == z[f"cb0{it}"].tolist()
    assert st.ctr.tolist() == z["final_ctr_t"].tolist()
    assert st.hist.tolist() == z["final_hist_t"].tolist()
    assert st.frames.tolist() == z["final_frames_t"].tolist()


def _depth_run(name, g, dtype, tag, greedy):
    z = golden(f"{name}_{dtype}.npz")
    W = {k: v.numpy() for k, v in WG.depth_weights(g).items()}
    d = DepthOracle(W, g, 3, dtype, temp=0.8, top_k=50, greedy=greedy)
    for s in range(3):
        d.set_speaker(s, z["mems"][s].reshape(-1), 1.0)
    d.row_seed[:3] = [11, 22, 2 ** 31 - 3]
    out = []
    for f in range(2):
        codes, fb = d.step(z["slots"], z[f"{tag}_h{f}"], z[f"{tag}_cb0_{f}"])
        out.append((codes, fb, z[f"{tag}_codes{f}"], z[f"{tag}_fb{f}"]))
    assert d.row_ctr.tolist() == z[f"{tag}_row_ctr"].tolist()
    return out


@pytest.mark.parametrize("greedy", [True, False])
def test_depth_fp32(greedy):
    for codes, fb, rc, rfb in _depth_run("depth_tiny", TINY.depth, "fp32", "g" if greedy else "s", greedy):
        assert (codes == rc).all()
        np.testing.assert_allclose(fb, rfb, atol=1e-5)


@pytest.mark.parametrize("greedy", [True, False])
def test_depth_bf16(greedy):
    """Greedy: bit-exact.  Sampled: a near-tie may flip under 1-ulp logit differences (one of 24 codes here)."""
    agree, total = 0, 0
    for codes, fb, rc, rfb in _depth_run("depth_tiny", TINY.depth, "bf16", "g" if greedy else "s", greedy):
        agree += int((codes == rc).sum())
        total += rc.size
        if (codes == rc).all():
            assert np.abs(fb - rfb).max() <= 2 ** -7 * max(1.0, np.abs(rfb).max())
    assert agree / total >= (1.0 if greedy else 0.9)


def test_depth_shared_groups_fp32():
    """n_q = 12 with levels 9-11 sharing one trunk: the incremental K/V branch of serve/fast_depth.py:169-173."""
    g = DepthGeom(layers=2, d=128, heads=2, ffn=256, n_q=12, rank=16, d_backbone=256)
    for greedy, tag in ((True, "g"), (False, "s")):
        for codes, fb, rc, rfb in _depth_run("depth_grouped", g, "fp32", tag, greedy):
            assert (codes == rc).all()
            np.testing.assert_allclose(fb, rfb, atol=1e-5)


@pytest.mark.parametrize("dtype,min_snr", [("fp32", 100.0), ("bf16", 35.0)])
def test_mimi(dtype, min_snr):
    g = TINY.mimi
    z = golden(f"mimi_tiny_{dtype}.npz")
    o = MimiOracle({k: v.numpy() for k, v in WG.mimi_weights(g).items()}, g, 3, dtype)
    got, ref = [], []
    for f in range(24):
        if f == 5:
            o.reset(2)
        if f == 14:
            o.reset(1)
        got.append(o.decode(z[f"slots{f}"], z[f"codes{f}"]))
        ref.append(z[f"pcm{f}"])
    got, ref = np.concatenate(got).astype(np.float64), np.concatenate(ref).astype(np.float64)
    snr = 10 * np.log10((ref ** 2).sum() / ((got - ref) ** 2).sum())
    assert snr > min_snr
