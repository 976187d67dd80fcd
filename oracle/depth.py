"""Whole-frame depth decoder -- TEST INFRASTRUCTURE (see oracle/__init__.py).

Restates ``FastDepth`` on its engine path (``fused=True``, per-row sampling streams): construction of the prefix
table and speaker constants (serve/fast_depth.py:43-82), the level loop ``_compute_fused`` (serve/fast_depth.py:143-203)
with ``add_ln`` (serve/fast_depth_kernels.py:271-302) and ``topk_sample`` (:305-336), and the backbone feedback embed
(tts/model/audio_io.py:27-35 as inlined at serve/fast_depth.py:200-202).
"""
import math

import numpy as np

from .common import Prec, f32, gelu, layer_norm, softmax
from .sampler import topk_sample


class DepthOracle:
    def __init__(self, weights, geom, max_slots, dtype="bf16", temp=0.7, top_k=64, greedy=False):
        self.g = g = geom
        self.rnd = rnd = Prec(dtype)
        self.max_slots = max_slots
        self.temp, self.top_k, self.greedy = float(temp), int(top_k), bool(greedy)
        W = {k: rnd(f32(v)) for k, v in weights.items()}
        self.W = W
        D, NL = g.d, g.n_q
        # prefix table: code_up(code_lo) + level_emb[1:], computed in the depth dtype (serve/fast_depth.py:49-50)
        table = rnd.mm(W["depth.code_lo.weight"], W["depth.code_up.weight"]).reshape(NL - 1, g.n_codes, D)
        self.embed = rnd(table + W["depth.level_emb.weight"][1:NL, None])
        self.level0 = W["depth.level_emb.weight"][0]
        self.cross = np.zeros((max_slots + 1, g.layers, D), np.float32)
        self.row_seed = np.zeros(max_slots + 1, np.int64)
        self.row_ctr = np.zeros(max_slots + 1, np.int64)

    def set_speaker(self, slot, mem, keep=1.0):
        """serve/fast_depth.py:72-82: one unmasked reference token, so cross-attention output = o(v(mem))."""
        D = self.g.d
        for li in range(self.g.layers):
            kv = self.rnd.mm(f32(mem).reshape(1, D), self.W[f"depth.cross.{li}.kv.weight"])
            v = self.rnd(kv[:, D:] * np.float32(keep))
            self.cross[slot, li] = self.rnd.mm(v, self.W[f"depth.cross.{li}.o.weight"])[0]

    def _add_ln(self, x, a, pre, c=None):
        x = self.rnd(x + a)
        if c is not None:
            x = self.rnd(x + c)
        return x, layer_norm(x, self.W[pre + "weight"], self.W[pre + "bias"], self.g.ln_eps, self.rnd)

    def _sdpa(self, q, k, v, causal):
        """q [B, H, Tq, hd], k/v [B, H, Tk, hd]; causal aligns the last query with the last key."""
        s = np.einsum("bhqd,bhkd->bhqk", q, k).astype(np.float32) * np.float32(self.g.head_dim ** -0.5)
        if causal:
            Tq, Tk = s.shape[-2:]
            mask = np.arange(Tk)[None, :] > (np.arange(Tq)[:, None] + (Tk - Tq))
            s = np.where(mask, np.float32(-np.inf), s)
        return self.rnd(np.einsum("bhqk,bhkd->bhqd", softmax(s), v))

    def step(self, slots, h, cb0, force=None):
        """FastDepth.__call__ -> (codes [B, n_q] int64, feedback [B, d_backbone]); advances row_ctr.

        force [B, n_q] (teacher forcing, for stage-by-stage comparisons): the next prefix rows and the feedback are
        built from these codes instead of the sampled ones; the sampled codes are still returned."""
        g, rnd, W = self.g, self.rnd, self.W
        slots = np.asarray(slots, np.int64)
        B, D, NL, H, HD, L = len(slots), g.d, g.n_q, g.heads, g.head_dim, g.layers
        cross = self.cross[slots]
        prefix = np.zeros((B, NL, D), np.float32)
        prefix[:, 0] = rnd(rnd.mm(h, W["depth.in_proj.weight"]) + self.level0)
        prefix[:, 1] = self.embed[0][np.asarray(cb0, np.int64)]
        kvbuf = [np.zeros((B, NL, 2, H, HD), np.float32) for _ in range(L)]
        codes = [np.asarray(cb0, np.int64)]
        previous = None
        seeds, ctrs = self.row_seed[slots], self.row_ctr[slots]
        self.last_logits = []
        for level in range(1, NL):
            group = g.group_of_level[level]
            n = level + 1
            incremental = group == previous
            reused_later = level + 1 < NL and g.group_of_level[level + 1] == group
            x = prefix[:, level:n] if incremental else prefix[:, :n]
            pre = f"depth.groups.{group}."
            y = layer_norm(x, W[pre + "0.n1.weight"], W[pre + "0.n1.bias"], g.ln_eps, rnd)
            for li in range(L):
                T = x.shape[1]
                qkv = rnd.mm(y, W[pre + f"{li}.qkv.weight"]).reshape(B, T, 3, H, HD)
                q = qkv[:, :, 0].transpose(0, 2, 1, 3)
                if incremental:
                    kvbuf[li][:, level:n] = qkv[:, :, 1:]
                    k = kvbuf[li][:, :n, 0].transpose(0, 2, 1, 3)
                    v = kvbuf[li][:, :n, 1].transpose(0, 2, 1, 3)
                    a = self._sdpa(q, k, v, causal=False)
                else:
                    if reused_later:
                        kvbuf[li][:, :n] = qkv[:, :, 1:]
                    k = qkv[:, :, 1].transpose(0, 2, 1, 3)
                    v = qkv[:, :, 2].transpose(0, 2, 1, 3)
                    if li == L - 1:
                        a = self._sdpa(q[:, :, -1:], k, v, causal=False)
                        x = x[:, -1:]
                    else:
                        a = self._sdpa(q, k, v, causal=True)
                T = x.shape[1]
                o = rnd.mm(a.transpose(0, 2, 1, 3).reshape(B, T, D), W[pre + f"{li}.o.weight"])
                x, y2 = self._add_ln(x, o, pre + f"{li}.n2.")
                f = rnd.mm(rnd(gelu(rnd.mm(y2, W[pre + f"{li}.f1.weight"]))), W[pre + f"{li}.f2.weight"])
                nxt = pre + f"{li + 1}.n1." if li + 1 < L else "depth.norm."
                x, y = self._add_ln(x, f, nxt, cross[:, li][:, None])
            logits = rnd.mm(y[:, -1], W[f"depth.heads.{level - 1}.weight"])
            self.last_logits.append(logits)
            code = topk_sample(logits, seeds, ctrs, level, self.temp, self.top_k, self.greedy)
            codes.append(code)
            used = code if force is None else np.asarray(force, np.int64)[:, level]
            if n < NL:
                prefix[:, n] = self.embed[level][used]
            previous = group
        np.add.at(self.row_ctr, slots, 1)
        codes = np.stack(codes, -1)
        return codes, self.feedback(codes if force is None else np.asarray(force, np.int64))

    def feedback(self, codes):
        """AudioInputEmbed.frames without its range check: RMSNorm(sum_k table[code_k + k*n_codes] / sqrt(n_q)),
        nn.RMSNorm(eps=None) -> fp32 epsilon."""
        g, rnd = self.g, self.rnd
        NL = codes.shape[1]
        e = self.W["audio_in.table.weight"][codes + np.arange(NL)[None] * g.n_codes]
        s = rnd(e.sum(1, dtype=np.float32))
        s = rnd(s / np.float32(math.sqrt(NL)))
        inv = np.float32(1) / np.sqrt((s * s).mean(-1, keepdims=True, dtype=np.float32) +
                                      np.float32(np.finfo(np.float32).eps))
        return rnd(s * inv * self.W["audio_in.norm.weight"])
