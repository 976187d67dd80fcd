"""configs[0] on the GPU: B = 4 seats, KV capacity 512, prompts torch.randint(0, 151936, (4, 200)) from generator
seed 0, 50 greedy frames with each frame's depth feedback fed back as the next backbone input (maya3/engine.py:
544-556), at the benchmark geometry (28-layer Qwen3-0.6B-class backbone, full vocabulary; 4 x 1024 depth stack with
8 codebooks; 8-codebook Mimi), through the native engine tick (TickEngine.tick: inline prefill of the 800 prompt rows
in the admission tick, then decode ticks).

Greedy: depth levels by argmax (FastDepth greedy), cb0 through the engine's own sampler at top-k 1 without the
presence penalty (Engine._cb0 with those settings is deterministic).  Stops are ignored (forced lengths).

Every tick is teacher-forced stage by stage against the oracle (the reference's arithmetic and bf16 rounding points,
pinned to fixtures made by running the reference): the backbone on the GPU's own input rows, the cb0 head and sampler
on the GPU's hidden state, each depth level from the GPU's own prefix, Mimi on the GPU's codes.  Per stage:
  * cb0 logits and every depth level's logits: max-abs difference <= 2e-2 of the logits' scale (bf16);
  * greedy codes: every disagreement is a near tie in the oracle's own logits (a few bf16 steps), and >= 98% agree;
  * PCM: SNR > 30 dB;
  * the backbone's hidden state: relative L2 below the 28-layer bf16 noise floor (5e-2)."""
import numpy as np
import pytest
import torch

from maya2_native_b200 import weights as WG
from maya2_native_b200.config import BASELINE
from maya2_native_b200.engine import TickConfig, TickEngine
from oracle.tick import OracleTick

pytestmark = pytest.mark.gpu
B, CAP, PROMPT, FRAMES = 4, 512, 200, 50


def snr_db(ref, x):
    return 10 * np.log10((ref ** 2).sum() / max(((ref - x) ** 2).sum(), 1e-30))


def scaled_maxabs(a, ref):
    return float(np.abs(np.asarray(a, np.float32) - ref).max() / max(1.0, float(np.abs(ref).max())))


def near_tie_gaps(lg, pick_ref, pick_gpu):
    """Relative gap, in the oracle's logits, between the oracle's pick and the GPU's pick of each flipped row."""
    out = []
    for r in np.nonzero(pick_ref != pick_gpu)[0]:
        a, b = float(lg[r, pick_ref[r]]), float(lg[r, pick_gpu[r]])
        out.append((a - b) / max(abs(a), 1e-30))
    return out


def test_config0_greedy_stage_parity(cuda):
    g = BASELINE
    Wt = WG.generate(WG.all_shapes(g), seed=0)
    Wn = {k: v.float().numpy() for k, v in Wt.items()}
    Wd = {k: v.to(cuda) for k, v in Wt.items()}
    del Wt
    cfg = TickConfig(max_seats=B, capacity=CAP, stops=False, greedy=True, cb0_top_k=1, cb0_rep=0.0, seed=7,
                     max_inline_rows=1024)
    eng = TickEngine(g, Wd, cfg, device=cuda)
    del Wd
    dbg = eng.depth.debug_logits()
    ora = OracleTick(Wn, g, B, CAP, "bf16", cb0_top_k=1, cb0_rep=0.0, cb0_rep_win=cfg.cb0_rep_win)
    ora.depth.greedy = True
    prompts = torch.randint(0, g.backbone.vocab, (B, PROMPT), generator=torch.Generator().manual_seed(0)).numpy()
    for i in range(B):
        eng.submit(prompts[i], max_frames=FRAMES + 4, seed=1000 + i)
    embed = ora.bb.rnd(Wn["model.embed_tokens.weight"])
    null_mem = Wn["depth.null_mem"]
    r = {"h_err": [], "cb0_logits": [], "depth_logits": [], "snr": [], "cb0_hit": 0, "code_hit": 0, "code_n": 0,
         "gaps": []}
    fb_prev = None
    for tick in range(FRAMES):
        out = eng.tick()
        order = [s for s, *_ in out]
        assert len(order) == B
        h_gpu, codes_gpu, pcm_gpu = (t.cpu() for t in eng.last_outputs(B))
        h_gpu = h_gpu.float().numpy()
        codes_gpu, pcm_gpu = codes_gpu.numpy(), pcm_gpu.numpy()
        cb0_gpu = np.array([c for _, _, c, _ in out], np.int64)
        lg_gpu = eng.cb0.copy_logits(B).float().cpu().numpy()
        dl_gpu = dbg[:, :B].float().cpu().numpy()
        slots = np.array([s.slot for s in order], np.int64)
        if tick == 0:
            for s in order:
                ora.st.min[s.slot] = cfg.min_frames
                ora.depth.set_speaker(s.slot, null_mem)
            _, last = ora.bb.step_mixed([], None, [(s.slot, embed[s.prompt]) for s in order])
            h_o = np.stack(last)
        else:
            h_o = ora.bb.step(list(slots), np.stack([fb_prev[int(sl)] for sl in slots]))
        r["h_err"].append(float(np.linalg.norm(h_o - h_gpu) / np.linalg.norm(h_o)))
        _, cb0_o, lg_o = ora.cb0(h_gpu, slots)
        r["cb0_logits"].append(scaled_maxabs(lg_gpu, lg_o))
        r["cb0_hit"] += int((cb0_o == cb0_gpu).sum())
        r["gaps"] += near_tie_gaps(lg_o[:, :2048], cb0_o, cb0_gpu)
        codes_o, fb_o = ora.depth.step(slots, h_gpu, cb0_gpu, force=codes_gpu)
        for lv in range(1, g.depth.n_q):
            lo = np.asarray(ora.depth.last_logits[lv - 1], np.float32)
            r["depth_logits"].append(scaled_maxabs(dl_gpu[lv - 1], lo))
            r["gaps"] += near_tie_gaps(lo, codes_o[:, lv], codes_gpu[:, lv])
        r["code_hit"] += int((codes_o[:, 1:] == codes_gpu[:, 1:]).sum())
        r["code_n"] += codes_o[:, 1:].size
        fb_gpu = eng.feedback[torch.from_numpy(slots).to(cuda)].float().cpu().numpy()
        r["snr"].append(float(snr_db(ora.mimi.decode(slots, codes_gpu), pcm_gpu)))
        fb_prev = {int(sl): fb_gpu[i] for i, sl in enumerate(slots)}
    assert eng.device_status() == 0
    eng.close()
    summary = {"h_err_max": max(r["h_err"]), "cb0_logits_max": max(r["cb0_logits"]),
               "depth_logits_max": max(r["depth_logits"]), "snr_min_db": min(r["snr"]),
               "cb0_agree": r["cb0_hit"] / (B * FRAMES), "depth_agree": r["code_hit"] / r["code_n"],
               "flips": len(r["gaps"]), "largest_flip_gap": max(r["gaps"], default=0.0)}
    print("configs[0] greedy stage parity:", summary)
    assert summary["cb0_logits_max"] <= 2e-2, summary
    assert summary["depth_logits_max"] <= 2e-2, summary
    assert summary["snr_min_db"] > 30, summary
    assert summary["h_err_max"] < 5e-2, summary
    assert summary["cb0_agree"] >= 0.98 and summary["depth_agree"] >= 0.98, summary
    assert summary["largest_flip_gap"] <= 2.0 ** -6, summary
