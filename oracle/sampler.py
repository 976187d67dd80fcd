"""cb0 sampler with controlled stop, and the depth top-k sampler -- TEST INFRASTRUCTURE (see oracle/__init__.py).

``cb0_sample`` restates ``Engine._cb0`` (maya3/engine.py:652-694) with ``row_exponential``
(serve/fast_depth_kernels.py:339-355); ``topk_sample`` restates ``_topk_sample`` (serve/fast_depth_kernels.py:305-336).
"""
import numpy as np

from .common import f32, softmax
from .philox import uniform

AEOS = 2048
STOP_ARGMAX, STOP_TAU, STOP_HAZARD = 2, 3, 4      # REASONS, maya3/engine.py:46


def _first_argmax(x):
    return np.argmax(x, -1).astype(np.int64)       # numpy returns the first index of the maximum, as torch/Triton


def topk_sample(logits, seeds, ctrs, level, temp, top_k, greedy=False):
    """logits [B, V] (the head output, any float) -> codes [B] int64.
    x = logits * (1/temp); kth = k-th largest; keep x >= kth; greedy: argmax; else argmax(x - log(-log u)) with
    u = tl.rand(seed_row, (ctr_row*32 + level)*V + c)."""
    x = f32(logits) * np.float32(1.0 / temp)
    B, V = x.shape
    kth = -np.sort(-x, axis=-1)[:, top_k - 1:top_k]
    xm = np.where(x >= kth, x, np.float32(-np.inf)).astype(np.float32)
    if greedy:
        return _first_argmax(xm)
    seeds = np.asarray(seeds, np.int64)[:, None]
    off = ((np.asarray(ctrs, np.int64) * 32 + level) * V)[:, None] + np.arange(V)[None]
    u = np.maximum(uniform(seeds, off), np.float32(1e-12))
    with np.errstate(divide="ignore"):
        score = xm - np.log(-np.log(u)).astype(np.float32)
    return _first_argmax(score)


def row_exponential(seeds, ctrs, V, level=0):
    off = ((np.asarray(ctrs, np.int64) * 32 + level) * 4096)[:, None] + np.arange(V)[None]
    u = np.maximum(uniform(np.asarray(seeds, np.int64)[:, None], off), np.float32(1e-12))
    return (-np.log(u)).astype(np.float32)


class Cb0State:
    """Per-slot sampler state of maya3/engine.py:210-223 (row max_slots is the padding slot)."""

    def __init__(self, max_slots, temp=0.9, top_k=64, top_p=1.0, rep=0.8, rep_win=12):
        m = max_slots + 1
        self.frames = np.zeros(m, np.int64)
        self.min = np.zeros(m, np.int64)
        self.hazard = np.zeros(m, np.float32)
        self.aeos_bias = np.zeros(m, np.float32)
        self.temp = np.full(m, temp, np.float32)
        self.topk = np.full(m, top_k, np.int64)
        self.topp = np.full(m, top_p, np.float32)
        self.rep = np.full(m, rep, np.float32)
        self.seed = np.zeros(m, np.int64)
        self.ctr = np.zeros(m, np.int64)
        self.hist = np.full((m, max(1, rep_win)), -1, np.int64)
        self.rep_win = rep_win


def cb0_sample(logits, idx, st, apply_rep=True, apply_top_p=None):
    """logits [B, 2049] as returned by the bf16 cb0 head -> (stop code [B], cb0 [B]); updates `st` like
    maya3/engine.py:689-693.  apply_rep mirrors `cb0_rep_win > 0 and (cb0_rep > 0 or any_rep)`, apply_top_p mirrors
    `_any_top_p` (default: any selected row has top_p < 1)."""
    idx = np.asarray(idx, np.int64)
    x = f32(logits) / st.temp[idx][:, None]
    x[:, AEOS] += st.aeos_bias[idx]
    if apply_rep and st.rep_win > 0:
        hist = st.hist[idx]
        pen = np.zeros_like(x)
        rows = np.repeat(np.arange(len(idx)), hist.shape[1])
        np.add.at(pen, (rows, np.maximum(hist, 0).ravel()), (hist >= 0).astype(np.float32).ravel())
        pen[:, AEOS] = 0
        x = (x - st.rep[idx][:, None] * (pen > 0).astype(np.float32)).astype(np.float32)
    srt = -np.sort(-x, axis=-1)
    k = np.clip(st.topk[idx] - 1, 0, x.shape[1] - 1)
    kth = srt[np.arange(len(idx)), k][:, None]
    x = np.where(x < kth, np.float32(-np.inf), x).astype(np.float32)
    if apply_top_p is None:
        apply_top_p = bool((st.topp[idx] < 1.0).any())
    if apply_top_p:
        p = softmax(x)
        order = np.argsort(-p, axis=-1, kind="stable")
        sp = np.take_along_axis(p, order, -1)
        drop = (np.cumsum(sp, -1, dtype=np.float32) - sp) > st.topp[idx][:, None]
        mask = np.zeros_like(drop)
        np.put_along_axis(mask, order, drop, -1)
        x = np.where(mask, np.float32(-np.inf), x).astype(np.float32)
    probs = softmax(x).astype(np.float32)
    pa = probs[:, AEOS]
    arg = _first_argmax(probs)
    frames = st.frames[idx]
    can = frames >= st.min[idx]
    hz = st.hazard[idx]
    hz = np.where(can, np.float32(1) - (np.float32(1) - hz) * (np.float32(1) - pa), hz).astype(np.float32)
    code = np.zeros(len(idx), np.int64)
    code = np.where(can & (hz >= np.float32(0.6)), STOP_HAZARD, code)
    code = np.where(can & (pa >= np.float32(0.35)), STOP_TAU, code)
    code = np.where(can & (arg == AEOS), STOP_ARGMAX, code)
    q = probs.copy()
    q[:, AEOS] = 0
    q = q / np.maximum(q.sum(-1, keepdims=True, dtype=np.float32), np.float32(1e-12))
    E = row_exponential(st.seed[idx], st.ctr[idx], q.shape[1], 0)
    cb0 = np.minimum(_first_argmax(q / E), AEOS - 1)
    st.ctr[idx] += 1
    if st.rep_win > 0:
        st.hist[idx] = np.concatenate([st.hist[idx, 1:], cb0[:, None]], 1)
    st.hazard[idx] = hz
    st.frames[idx] = frames + 1
    return code, cb0
