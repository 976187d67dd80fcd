"""GPU parity of the samplers: the depth top-k sampler and the cb0 sampler with controlled stop, against fixtures
produced by the reference's own Triton kernels and Engine._cb0 (tests/golden/make_golden.py).

The noise is the same counter-based Philox stream as the reference's tl.rand, so given identical logits the sampled
codes are expected to be identical, not just equal in distribution."""
import numpy as np
import pytest
import torch

from conftest import golden
from maya2_native_b200 import weights as WG
from maya2_native_b200.config import TINY
from maya2_native_b200.sampler import Cb0Sampler, topk_sample

pytestmark = pytest.mark.gpu


def test_topk_sampler_bit_exact(cuda):
    z = golden("topk_sampler.npz")
    lg = torch.from_numpy(z["logits"]).to(cuda)
    seeds, ctrs = torch.from_numpy(z["seeds"]), torch.from_numpy(z["ctrs"])
    for level in (1, 5, 31):
        for k in (1, 50, 64, 2048):
            got = topk_sample(lg, seeds, ctrs, level, 0.7, k).cpu().numpy()
            assert (got == z[f"s_l{level}_k{k}"]).all(), (level, k)
        got = topk_sample(lg, seeds, ctrs, level, 0.8, 50, greedy=True).cpu().numpy()
        assert (got == z[f"g_l{level}"]).all()
    lb = torch.from_numpy(z["logits_bf16"]).to(cuda, torch.bfloat16)
    assert (topk_sample(lb, seeds, ctrs, 3, 0.8, 50).cpu().numpy() == z["s_bf16"]).all()


def test_topk_sampler_distribution(cuda):
    """serve/../test_depth_fused.py:9-23: total variation vs the exact top-k softmax < 0.03 over 200k draws."""
    g = torch.Generator().manual_seed(0)
    lg = (torch.randn(1, 2048, generator=g) * 3).to(cuda)
    rows = 4000
    draws = []
    for i in range(50):
        seeds = torch.arange(rows, dtype=torch.int32) + i * rows
        draws.append(topk_sample(lg.expand(rows, -1).contiguous(), seeds, torch.zeros(rows, dtype=torch.int32), 3,
                                 0.7, 64))
    d = torch.cat(draws)
    emp = torch.bincount(d, minlength=2048).float() / d.numel()
    x = lg[0] / 0.7
    kth = x.topk(64).values[-1]
    p = torch.where(x >= kth, x, torch.tensor(-float("inf"), device=cuda)).softmax(-1)
    tv = 0.5 * (emp - p).abs().sum().item()
    assert tv < 0.03
    assert emp[p == 0].sum().item() == 0


def _sampler_from_fixture(z, cuda, g):
    s = Cb0Sampler(WG.make("cb0_head.weight", (g.n_cb0, g.hidden)), 5, max_rows=8, device=cuda)
    for name in ("temp_t", "topk_t", "topp_t", "rep_t", "aeos_bias", "seed_t", "ctr_t", "hist_t", "frames_t",
                 "min_t", "hazard_t"):
        getattr(s, name).copy_(torch.from_numpy(z["init_" + name]))
    s.any_rep = True
    s.any_top_p = True
    return s


def test_cb0_sampler_matches_engine_on_fixture_logits(cuda):
    g = TINY.backbone
    z = golden("cb0_sampler.npz")
    s = _sampler_from_fixture(z, cuda, g)
    idx = torch.arange(5, device=cuda)
    for it in range(3):
        code, cb0 = s.sample_logits(torch.from_numpy(z[f"logits{it}"]), idx)
        assert code.cpu().tolist() == z[f"code{it}"].tolist(), it
        assert cb0.cpu().tolist() == z[f"cb0{it}"].tolist(), it
    assert s.ctr_t.cpu().tolist() == z["final_ctr_t"].tolist()
    assert s.hist_t.cpu().tolist() == z["final_hist_t"].tolist()
    assert s.frames_t.cpu().tolist() == z["final_frames_t"].tolist()
    np.testing.assert_allclose(s.hazard_t.cpu().numpy(), z["final_hazard_t"], rtol=1e-6, atol=1e-7)


def test_cb0_step_from_hidden_states(cuda):
    """Head GEMM + sampler from h: the bf16 logits may differ from the reference's GEMM by an ulp, so allow one
    sampled code to move."""
    g = TINY.backbone
    z = golden("cb0_sampler.npz")
    s = _sampler_from_fixture(z, cuda, g)
    idx = torch.arange(5, device=cuda)
    miss = 0
    for it in range(3):
        h = torch.from_numpy(z[f"h{it}"]).to(cuda, torch.bfloat16)
        code, cb0 = s(h, idx)
        assert code.cpu().tolist() == z[f"code{it}"].tolist()
        miss += int((cb0.cpu().numpy() != z[f"cb0{it}"]).sum())
    assert miss <= 1
