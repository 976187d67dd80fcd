"""Tick-level parity: the native engine tick (m3_tick_run from a CUDA graph) against the CPU oracle composed the way
Engine._tick composes its stages (maya3/engine.py:534-563), teacher-forced stage by stage.

Per tick and seat the oracle runs each stage on the GPU's own inputs to that stage -- the backbone on the GPU's
feedback vector (the prompt's embeddings on the admission tick), cb0 on the GPU's hidden state, the depth loop on the
GPU's cb0 with the GPU's codes as the prefix, Mimi on the GPU's codes -- so every comparison measures one stage of
one tick while the caches (backbone KV, Mimi ring and conv state, sampler counters) evolve in both from the same
inputs.  Random-init TINY geometry, sampled decoding with per-seat Philox streams; the oracle emulates the
reference's bf16 rounding points.  Thresholds follow the reference's own tests (sampler agreement, relative error
of the hidden state, PCM SNR)."""
import numpy as np
import pytest
import torch

from maya2_native_b200 import weights as WG
from maya2_native_b200.config import TINY
from maya2_native_b200.engine import TickConfig, TickEngine
from oracle.tick import OracleTick

pytestmark = pytest.mark.gpu


def snr_db(ref, x):
    return 10 * np.log10((ref ** 2).sum() / max(((ref - x) ** 2).sum(), 1e-30))


def test_tick_matches_oracle_stage_by_stage(cuda):
    g = TINY
    Wt = WG.generate(WG.all_shapes(g), seed=0)
    Wn = {k: v.float().numpy() for k, v in Wt.items()}
    Wd = {k: v.to(cuda) for k, v in Wt.items()}
    cfg = TickConfig(max_seats=4, capacity=256, stops=False, seed=7, max_inline_rows=64)
    eng = TickEngine(g, Wd, cfg, device=cuda)
    ora = OracleTick(Wn, g, 4, 256, "bf16", temp=cfg.temp, top_k=cfg.top_k, cb0_temp=cfg.cb0_temp,
                     cb0_top_k=cfg.cb0_top_k, cb0_rep=cfg.cb0_rep, cb0_rep_win=cfg.cb0_rep_win)
    rng = np.random.default_rng(0)
    lens = (7, 12, 5, 20)
    seats = [eng.submit(rng.integers(0, g.backbone.vocab, n), max_frames=24, seed=1000 + i)
             for i, n in enumerate(lens)]
    null_mem = Wn["depth.null_mem"]
    embed = ora.bb.rnd(Wn["model.embed_tokens.weight"])

    h_err, cb0_hit, cb0_n, code_hit, code_n, fb_err, snrs = [], 0, 0, 0, 0, [], []
    for tick in range(16):
        dec = list(eng.active)
        out = eng.tick()
        order = [s for s, *_ in out]
        assert len(order) == 4
        h_gpu, codes_gpu, pcm_gpu = (t.cpu() for t in eng.last_outputs(4))
        h_gpu = h_gpu.float().numpy()
        codes_gpu, pcm_gpu = codes_gpu.numpy(), pcm_gpu.numpy()
        cb0_gpu = np.array([c for _, _, c, _ in out], np.int64)
        assert (codes_gpu[:, 0] == cb0_gpu).all()
        slots = np.array([s.slot for s in order], np.int64)
        if tick == 0:
            assert not dec
            for s in order:        # the seat state a bind installs (maya3/engine.py:420-447)
                ora.st.seed[s.slot] = s.seed
                ora.st.min[s.slot] = cfg.min_frames
                ora.depth.row_seed[s.slot] = (s.seed * 69069 + 1) % (2 ** 31 - 1)
                ora.depth.set_speaker(s.slot, null_mem)
            _, last = ora.bb.step_mixed([], None, [(s.slot, embed[s.prompt]) for s in order])
            h_o = np.stack(last)
        else:
            h_o = ora.bb.step(list(slots), fb_prev)
        h_err.append(np.linalg.norm(h_o - h_gpu) / np.linalg.norm(h_o))
        code, cb0_o, _ = ora.cb0(h_gpu, slots)
        cb0_hit += int((cb0_o == cb0_gpu).sum())
        cb0_n += len(slots)
        ora.st.hist[slots, -1] = cb0_gpu                 # keep the repetition window on the GPU's trajectory
        codes_o, fb_o = ora.depth.step(slots, h_gpu, cb0_gpu, force=codes_gpu)
        code_hit += int((codes_o[:, 1:] == codes_gpu[:, 1:]).sum())
        code_n += codes_o[:, 1:].size
        fb_gpu = eng.feedback[torch.from_numpy(slots).to(cuda)].float().cpu().numpy()
        fb_err.append(np.abs(fb_o - fb_gpu).max())
        pcm_o = ora.mimi.decode(slots, codes_gpu)
        snrs.append(snr_db(pcm_o, pcm_gpu))
        fb_prev = fb_gpu

    assert eng.device_status() == 0
    assert max(h_err) < 2e-2, h_err
    assert cb0_hit / cb0_n >= 0.9, (cb0_hit, cb0_n)
    assert code_hit / code_n >= 0.9, (code_hit, code_n)
    assert max(fb_err) < 5e-2, fb_err
    assert min(snrs) > 30, snrs
    eng.close()
