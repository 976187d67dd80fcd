"""Backbone decode over the static per-seat KV cache -- TEST INFRASTRUCTURE (see oracle/__init__.py).

Restates ``StaticBackbone._forward`` on its engine path (``fuse_rope=True, attention='triton'``,
serve/fast_backbone.py:176-234) with the three Triton kernels it calls:
  * ``_add_rms``           serve/fast_backbone.py:96-104   h' = h + a ; y = w * bf16(h' / rms(h'))
  * ``_qk_norm_rope_cache`` serve/fast_backbone.py:62-92   q/k head RMSNorm + RoPE in fp32 + K/V cache write
  * ``_decode_attn``       serve/fast_backbone.py:32-58    attention of each row over keys 0..pos of its slot
In fp32 the same function reduces to the reference's ``attention='gather'`` path (serve/fast_backbone.py:204-228).
"""
import numpy as np

from .common import Prec, f32, silu


def inv_freq(head_dim, theta, rnd):
    """HF default RoPE frequencies 1/theta^(2i/d).  The reference casts the whole model to its serving dtype
    (tts/model/load_s3.py:417-419), which rounds this buffer too, so it is stored through ``rnd``."""
    inv = (1.0 / (np.float32(theta) ** (np.arange(0, head_dim, 2, dtype=np.int64).astype(np.float32) /
                                         np.float32(head_dim)))).astype(np.float32)
    return rnd(inv)


def rope_tables(head_dim, capacity, theta, rnd):
    """Qwen3RotaryEmbedding: emb = [f, f] with f = pos * inv_freq in fp32; cos/sin in fp32."""
    inv = inv_freq(head_dim, theta, rnd)
    f = np.arange(capacity, dtype=np.float32)[:, None] * inv[None, :]
    emb = np.concatenate([f, f], -1).astype(np.float32)
    return np.cos(emb).astype(np.float32), np.sin(emb).astype(np.float32)


class BackboneOracle:
    """Owns the static cache [layers, max_slots+1, kv_heads, capacity, head_dim] (row max_slots = dummy) and
    per-slot lengths, exactly as StaticBackbone.__init__ (serve/fast_backbone.py:146-153)."""

    def __init__(self, weights, geom, max_slots, capacity, dtype="bf16"):
        self.g = g = geom
        self.rnd = Prec(dtype)
        self.max_slots, self.capacity, self.dummy = max_slots, capacity, max_slots
        W = {k: self.rnd(f32(v)) for k, v in weights.items() if not k.startswith("model.embed_tokens")}
        self.embed = weights.get("model.embed_tokens.weight")
        self.layers = []
        for i in range(g.layers):
            p = f"model.layers.{i}."
            self.layers.append(dict(
                in_ln=W[p + "input_layernorm.weight"], post_ln=W[p + "post_attention_layernorm.weight"],
                wqkv=np.concatenate([W[p + "self_attn.q_proj.weight"], W[p + "self_attn.k_proj.weight"],
                                     W[p + "self_attn.v_proj.weight"]], 0),
                q_norm=W[p + "self_attn.q_norm.weight"], k_norm=W[p + "self_attn.k_norm.weight"],
                wo=W[p + "self_attn.o_proj.weight"],
                wgu=np.concatenate([W[p + "mlp.gate_proj.weight"], W[p + "mlp.up_proj.weight"]], 0),
                wd=W[p + "mlp.down_proj.weight"]))
        self.norm_w = W["model.norm.weight"]
        self.cb0_w = W["cb0_head.weight"]
        cos, sin = rope_tables(g.head_dim, capacity, g.rope_theta, self.rnd)
        self.cos, self.sin = self.rnd(cos), self.rnd(sin)          # model dtype, as HF returns them
        shape = (g.layers, max_slots + 1, g.kv_heads, capacity, g.head_dim)
        self.k = np.zeros(shape, np.float32)
        self.v = np.zeros(shape, np.float32)
        self.lengths = np.zeros(max_slots + 1, np.int64)

    # ---------------------------------------------------------------- pieces
    def _rms(self, x, w):
        """Qwen3RMSNorm: w * bf16(x * 1/sqrt(mean(x^2) + eps)) in fp32, stored once."""
        x = f32(x)
        inv = np.float32(1.0) / np.sqrt((x * x).mean(-1, keepdims=True, dtype=np.float32) + np.float32(self.g.eps))
        return self.rnd(self.rnd(x * inv) * w)

    def _add_rms(self, h, a, w):
        h = self.rnd(f32(h) + f32(a))
        return h, self._rms(h, w)

    def _qk_rope(self, x, w, pos):
        """x [B, n, D] -> head RMSNorm + rotate-half RoPE at pos [B] (fp32 math, one rounding)."""
        y = self._rms(x, w)
        half = self.g.head_dim // 2
        c, s = self.cos[pos][:, None], self.sin[pos][:, None]
        y1, y2 = y[..., :half], y[..., half:]
        o1 = y1 * c[..., :half] - y2 * s[..., :half]
        o2 = y2 * c[..., half:] + y1 * s[..., half:]
        return self.rnd(np.concatenate([o1, o2], -1))

    def _attend(self, q, kc, vc, slot, pos):
        """q [H, D] of one row over keys 0..pos of `slot` (GQA: head h reads kv head h // G)."""
        g = self.g
        G = g.groups
        K = kc[slot, :, :pos + 1]               # [KV, T, D]
        V = vc[slot, :, :pos + 1]
        qh = q.reshape(g.kv_heads, G, g.head_dim)
        s = np.einsum("kgd,ktd->kgt", qh, K).astype(np.float32) * np.float32(g.head_dim ** -0.5)
        m = s.max(-1, keepdims=True)
        p = np.exp(s - m)
        o = np.einsum("kgt,ktd->kgd", p, V) / p.sum(-1, keepdims=True)
        return self.rnd(o.reshape(g.heads, g.head_dim))

    # ---------------------------------------------------------------- step
    def forward(self, slots, x, offsets=None, real=None):
        """One decode (or mixed decode + inline prefill) step; serve/fast_backbone.py:176-234.

        slots [R] (prefill rows repeat their slot), x [R, hidden], offsets [R] (position offset of each prefill
        row; 0 for decode rows), real [R] (1 for rows that advance their slot's length).  Returns the final-normed
        hidden state [R, hidden]."""
        g = self.g
        slots = np.asarray(slots, np.int64)
        R = len(slots)
        pos = self.lengths[slots] + (np.asarray(offsets, np.int64) if offsets is not None else 0)
        H, KV, D = g.heads, g.kv_heads, g.head_dim
        h = self.rnd(x)
        pend = None
        for i, L in enumerate(self.layers):
            if pend is not None:
                h, y = self._add_rms(h, pend, L["in_ln"])
            else:
                y = self._rms(h, L["in_ln"])
            qkv = self.rnd.mm(y, L["wqkv"])
            q = self._qk_rope(qkv[:, :H * D].reshape(R, H, D), L["q_norm"], pos)
            k = self._qk_rope(qkv[:, H * D:(H + KV) * D].reshape(R, KV, D), L["k_norm"], pos)
            v = qkv[:, (H + KV) * D:].reshape(R, KV, D)
            kc, vc = self.k[i], self.v[i]
            kc[slots, :, pos] = k                  # every row writes its K/V before any row attends
            vc[slots, :, pos] = v
            o = np.stack([self._attend(q[r], kc, vc, slots[r], pos[r]) for r in range(R)])
            a = self.rnd.mm(o.reshape(R, H * D), L["wo"])
            h, y2 = self._add_rms(h, a, L["post_ln"])
            gu = self.rnd.mm(y2, L["wgu"])
            act = self.rnd(self.rnd(silu(gu[:, :g.ffn])) * gu[:, g.ffn:])
            pend = self.rnd.mm(act, L["wd"])
        h, out = self._add_rms(h, pend, self.norm_w)
        np.add.at(self.lengths, slots, np.ones(R, np.int64) if real is None else np.asarray(real, np.int64))
        return out

    def step(self, slots, x):
        """StaticBackbone.step (serve/fast_backbone.py:289-315): one decode row per distinct slot."""
        if len(set(slots)) != len(slots):
            raise ValueError("duplicate slots in one step")
        return self.forward(slots, x)

    def step_mixed(self, slots, x, prefills):
        """StaticBackbone.step_mixed (serve/fast_backbone.py:326-359): decode rows plus T consecutive rows per
        inline prefill.  Returns (decoded [B, hidden], [last hidden per prefill])."""
        index, offsets, rows = list(slots), [0] * len(slots), [] if x is None else [f32(x)]
        for s, t in prefills:
            index += [s] * len(t)
            offsets += list(range(len(t)))
            rows.append(f32(t))
        out = self.forward(index, np.concatenate(rows, 0), offsets)
        last, at = [], len(slots)
        for _, t in prefills:
            at += len(t)
            last.append(out[at - 1])
        return out[:len(slots)], last

    def load_slot(self, slot, keys, values, length):
        """Install per-layer K/V [layers, KV, length, D] for a slot (serve/fast_backbone.py:158-165)."""
        self.k[:, slot, :, :length] = keys
        self.v[:, slot, :, :length] = values
        self.lengths[slot] = length

    def free(self, slot):
        self.lengths[slot] = 0

    def cb0_logits(self, h):
        """Backbone.cb0_logits (tts/model/backbone.py:97): the cb0 head Linear in the model dtype, as fp32."""
        return self.rnd.mm(h, self.cb0_w)
