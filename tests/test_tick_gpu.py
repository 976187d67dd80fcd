"""Tick-level parity: the native engine tick (m3_tick_run from a CUDA graph) against the CPU oracle composed the way
Engine._tick composes its stages (maya3/engine.py:534-563), teacher-forced stage by stage.

Per tick and seat the oracle runs each stage on the GPU's own inputs to that stage -- the backbone on the GPU's
feedback vector (the prompt's embeddings on the admission tick), cb0 on the GPU's hidden state, the depth loop on the
GPU's cb0 with the GPU's codes as the prefix, Mimi on the GPU's codes -- so every comparison measures one stage of
one tick while the caches (backbone KV, Mimi ring and conv state, sampler counters) evolve in both from the same
inputs.  Random-init weights, sampled decoding with per-seat Philox streams; the oracle emulates the reference's
bf16 rounding points.  Thresholds follow the reference's own tests (sampler agreement, relative error of the hidden
state, PCM SNR)."""
import dataclasses

import numpy as np
import pytest
import torch

from maya2_native_b200 import weights as WG
from maya2_native_b200.config import BASELINE, TINY
from maya2_native_b200.engine import TickConfig, TickEngine
from oracle.tick import OracleTick

pytestmark = pytest.mark.gpu


def snr_db(ref, x):
    return 10 * np.log10((ref ** 2).sum() / max(((ref - x) ** 2).sum(), 1e-30))


def run_stage_parity(g, cuda, lens, ticks, capacity, max_inline=None):
    Wt = WG.generate(WG.all_shapes(g), seed=0)
    Wn = {k: v.float().numpy() for k, v in Wt.items()}
    Wd = {k: v.to(cuda) for k, v in Wt.items()}
    del Wt
    n = len(lens)
    cfg = TickConfig(max_seats=n, capacity=capacity, stops=False, seed=7,
                     max_inline_rows=max_inline or max(64, sum(lens)))
    eng = TickEngine(g, Wd, cfg, device=cuda)
    del Wd
    ora = OracleTick(Wn, g, n, capacity, "bf16", temp=cfg.temp, top_k=cfg.top_k, cb0_temp=cfg.cb0_temp,
                     cb0_top_k=cfg.cb0_top_k, cb0_rep=cfg.cb0_rep, cb0_rep_win=cfg.cb0_rep_win)
    rng = np.random.default_rng(0)
    for i, m in enumerate(lens):
        eng.submit(rng.integers(0, g.backbone.vocab, m), max_frames=ticks + 4, seed=1000 + i)
    null_mem = Wn["depth.null_mem"]
    embed = ora.bb.rnd(Wn["model.embed_tokens.weight"])
    res = {"h_err": [], "cb0_hit": 0, "cb0_n": 0, "code_hit": 0, "code_n": 0, "fb_err": [], "snr": [],
           "cb0_logits": []}
    fb_prev = None
    for tick in range(ticks):
        dec = list(eng.active)
        out = eng.tick()
        order = [s for s, *_ in out]
        assert len(order) == n
        h_gpu, codes_gpu, pcm_gpu = (t.cpu() for t in eng.last_outputs(n))
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
        else:   # each seat's own feedback vector from the previous tick
            h_o = ora.bb.step(list(slots), np.stack([fb_prev[int(sl)] for sl in slots]))
        res["h_err"].append(float(np.linalg.norm(h_o - h_gpu) / np.linalg.norm(h_o)))
        lg_gpu = eng.cb0.copy_logits(n).float().cpu().numpy()
        _, cb0_o, lg_o = ora.cb0(h_gpu, slots)
        res["cb0_logits"].append(float(np.abs(lg_gpu - lg_o).max() / max(1.0, float(np.abs(lg_o).max()))))
        res["cb0_hit"] += int((cb0_o == cb0_gpu).sum())
        res["cb0_n"] += len(slots)
        ora.st.hist[slots, -1] = cb0_gpu                 # keep the repetition window on the GPU's trajectory
        codes_o, fb_o = ora.depth.step(slots, h_gpu, cb0_gpu, force=codes_gpu)
        res["code_hit"] += int((codes_o[:, 1:] == codes_gpu[:, 1:]).sum())
        res["code_n"] += codes_o[:, 1:].size
        fb_gpu = eng.feedback[torch.from_numpy(slots).to(cuda)].float().cpu().numpy()
        res["fb_err"].append(float(np.abs(fb_o - fb_gpu).max()))
        pcm_o = ora.mimi.decode(slots, codes_gpu)
        res["snr"].append(float(snr_db(pcm_o, pcm_gpu)))
        fb_prev = {int(sl): fb_gpu[i] for i, sl in enumerate(slots)}
    assert eng.device_status() == 0
    res["eager_prefill_rows"] = eng.stats["eager_prefill_rows"]
    eng.close()
    return res


def test_tick_matches_oracle_stage_by_stage(cuda):
    r = run_stage_parity(TINY, cuda, (7, 12, 5, 20), 16, 256)
    assert max(r["h_err"]) < 2e-2, r
    assert r["cb0_hit"] / r["cb0_n"] >= 0.9, r
    assert r["code_hit"] / r["code_n"] >= 0.9, r
    assert max(r["fb_err"]) < 5e-2, r
    assert max(r["cb0_logits"]) <= 2e-2, r
    assert min(r["snr"]) > 30, r


def test_tick_benchmark_geometry_stage_by_stage(cuda):
    """The same at the benchmark geometry (28-layer backbone, 4-layer x 8-codebook depth, Mimi with the fused SEANet
    stages); vocabulary reduced to 4096 ids (the embedding gather is width-independent).  After 28 bf16 layers the
    GPU and the bf16-emulating oracle differ only by accumulation order."""
    g = dataclasses.replace(BASELINE, backbone=dataclasses.replace(BASELINE.backbone, vocab=4096))
    r = run_stage_parity(g, cuda, (24, 40, 16, 56), 6, 512)
    print("benchmark-geometry stage parity:", r)
    assert max(r["h_err"]) < 5e-2, r
    assert r["cb0_hit"] / r["cb0_n"] >= 0.85, r
    assert r["code_hit"] / r["code_n"] >= 0.85, r
    assert max(r["fb_err"]) < 1e-1, r
    assert max(r["cb0_logits"]) <= 2e-2, r
    assert min(r["snr"]) > 30, r


def test_tick_eager_prefill_of_a_long_prompt(cuda):
    """A prompt longer than the tick's row budget: its head is prefilled by eager chunked backbone steps and its tail
    rides the admission tick inline (the reference's fallback prefill); the oracle prefills the whole prompt at once."""
    r = run_stage_parity(TINY, cuda, (40, 7), 6, 256, max_inline=16)
    assert r["eager_prefill_rows"] == 24, r
    assert max(r["h_err"]) < 2e-2, r
    assert r["cb0_hit"] / r["cb0_n"] >= 0.9, r
    assert min(r["snr"]) > 30, r


def test_stop_code_releases_the_seat(cuda):
    """Controlled stop through the engine loop (maya3/engine.py:565-635): a seat whose AEOS logit is biased up stops
    once it has its minimum frames, its last readout row carries the stop code and no PCM, its slot is released and
    the waiting request takes it on a following tick; the other seat keeps decoding."""
    W = WG.generate(WG.all_shapes(TINY))
    cfg = TickConfig(max_seats=2, capacity=64, max_inline_rows=16)
    eng = TickEngine(TINY, W, cfg, device=cuda)
    rng = np.random.default_rng(0)
    a, b, c = (eng.submit(rng.integers(0, TINY.backbone.vocab, 6), 30, seed=11 + i) for i in range(3))
    eng.tick()
    assert {a.slot, b.slot} == {0, 1} and c in eng.pending
    slot_a = a.slot
    with torch.inference_mode():
        eng.cb0.aeos_bias[slot_a] = 1e4
    stop_row = None
    for _ in range(cfg.min_frames + 4):
        for s, code, _, pcm in eng.tick():
            if s is a and code:
                stop_row = (code, pcm)
        if stop_row:
            break
    assert stop_row is not None and stop_row[1] is None
    assert a.stop in ("aeos", "aeos_argmax", "aeos_tau", "aeos_hazard") and a.frames >= cfg.min_frames - 1
    assert a not in eng.active and b in eng.active and b.stop is None
    for _ in range(2):
        eng.tick()
    assert c in eng.active and c.slot == slot_a and c.frames >= 1
    assert eng.device_status() == 0
    eng.close()


def test_voice_prefix_request(cuda):
    """prepare_voice + submit(voice=...) (maya3/engine.py:259-283, :488-491): the request's slot starts from the
    voice's K/V (bit-identical to its store) and the prompt follows it; the first frame's hidden state matches a
    request that prefills prefix + prompt inline in the same tick."""
    W = WG.generate(WG.all_shapes(TINY))
    cfg = TickConfig(max_seats=2, capacity=128, max_inline_rows=64, stops=False)
    eng = TickEngine(TINY, W, cfg, device=cuda)
    rng = np.random.default_rng(9)
    pre, prompt = rng.integers(0, TINY.backbone.vocab, 20), rng.integers(0, TINY.backbone.vocab, 7)
    v = eng.prepare_voice(pre)
    a = eng.submit(prompt, 10, seed=5, voice=v)
    b = eng.submit(np.concatenate([pre, prompt]), 10, seed=5)
    eng.tick()
    assert eng.backbone.lengths_cpu[a.slot] == eng.backbone.lengths_cpu[b.slot] == 27
    assert eng.backbone.lengths.cpu().tolist()[a.slot] == 27
    for i in range(TINY.backbone.layers):
        assert torch.equal(eng.backbone.k[i][a.slot, :, :20], v.store[i, 0])
        assert torch.equal(eng.backbone.v[i][a.slot, :, :20], v.store[i, 1])
    h, _, _ = eng.last_outputs(2)
    h = h.float().cpu().numpy()
    assert np.abs(h[0] - h[1]).max() / max(1.0, np.abs(h[1]).max()) < 2e-2
    long_prompt = rng.integers(0, TINY.backbone.vocab, 100)
    eng.submit(long_prompt, 10)                            # fits alone: 100 + 10 + 2 <= 128
    with pytest.raises(ValueError):
        eng.submit(long_prompt, 10, voice=v)               # the prefix counts: a budget under 8 frames is refused
    assert eng.device_status() == 0
    eng.close()
