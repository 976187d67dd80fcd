"""One-frame streaming Mimi decoder -- TEST INFRASTRUCTURE (see oracle/__init__.py).

Restates ``StaticMimi`` (serve/fast_codec.py): per-slot conv histories and transposed-conv overlap tails
(``_layer`` :104-132), the split RVQ decode (``_quantizer``/``_rvq`` :134-149), the upsample, and the sliding-window
decoder transformer over a per-slot KV ring with absolute key positions (``_transformer`` :151-184).  Module math
follows HF MimiModel (transformers models/mimi/modeling_mimi.py: MimiConv1d, MimiConvTranspose1d, MimiResnetBlock,
MimiTransformerLayer, apply_rotary_pos_emb).  Arrays are channels-first [B, C, L] like the reference.
"""
import numpy as np

from maya2_native_b200.weights import mimi_decoder_layout

from .backbone import inv_freq
from .common import Prec, elu, f32, gelu, layer_norm, softmax

NEVER = -(1 << 40)


class MimiOracle:
    def __init__(self, weights, geom, max_slots, dtype="bf16"):
        self.g = g = geom
        self.rnd = rnd = Prec(dtype)
        self.max_slots, self.dummy = max_slots, max_slots
        self.W = W = {k[len("mimi."):]: rnd(f32(v)) for k, v in weights.items() if k.startswith("mimi.")}
        rows = max_slots + 1
        self.layout = mimi_decoder_layout(g)
        # stateful layers -> (channels, columns) as StaticMimi._plan (serve/fast_codec.py:81-96)
        self.state = {"upsample": np.zeros((rows, g.hidden, g.upsample_stride), np.float32)}
        for idx, kind, cin, cout, k, stride in self.layout:
            if kind == "conv" and k > 1:
                self.state[f"decoder.{idx}"] = np.zeros((rows, cin, k - 1), np.float32)
            elif kind == "convt":
                self.state[f"decoder.{idx}"] = np.zeros((rows, cout, stride), np.float32)
            elif kind == "resnet":
                self.state[f"decoder.{idx}.block.1"] = np.zeros((rows, cin, k - 1), np.float32)
        self.kv = np.zeros((g.layers, 2, rows, g.heads, g.ring, g.head_dim), np.float32)
        self.key_pos = np.full((rows, g.ring), NEVER, np.int64)
        self.tokens = np.zeros(rows, np.int64)
        self.inv_freq = inv_freq(g.head_dim, g.rope_theta, rnd)     # buffer in the model dtype, as StaticMimi reads it

    def reset(self, slot):
        """StaticMimi.reset (serve/fast_codec.py:231-244)."""
        for s in self.state.values():
            s[slot] = 0
        self.key_pos[slot] = NEVER
        self.tokens[slot] = 0

    # ---------------------------------------------------------------- layers
    def _conv(self, x, key, slots, w, b):
        """Stride-1 causal conv; the layer's history (if any) is prepended and refreshed."""
        k = w.shape[2]
        if key in self.state:
            st = self.state[key]
            x = np.concatenate([st[slots], x], -1)
            st[slots] = x[..., -st.shape[-1]:]
        L = x.shape[-1] - (k - 1)
        y = sum(np.einsum("oc,bcl->bol", w[:, :, j], x[..., j:j + L]) for j in range(k))
        return self.rnd(y + (b[None, :, None] if b is not None else 0))

    def _convt(self, x, key, slots, w, b, stride, groups=1):
        """ConvTranspose1d with the overlap tail kept per slot, bias removed from the stored tail."""
        B, C, L = x.shape
        k = w.shape[2]
        if groups == 1:
            z = np.einsum("bcl,cok->bolk", x, w)             # [B, Cout, L, k]
        else:
            z = x[:, :, :, None] * w[None, :, 0, None, :]    # depthwise: [B, C, L, k]
        cout = z.shape[1]
        y = np.zeros((B, cout, (L - 1) * stride + k), np.float32)
        for t in range(L):
            y[..., t * stride:t * stride + k] += z[:, :, t]
        y = self.rnd(y + (b[None, :, None] if b is not None else 0))
        produced = L * stride
        st = self.state[key]
        prev = st[slots].copy()
        tail = y[..., produced:]
        if b is not None:
            tail = self.rnd(tail - b[None, :, None])
        st[slots] = tail
        ov = st.shape[-1]
        y[..., :ov] = self.rnd(y[..., :ov] + prev)
        return y[..., :produced]

    def _quantizer(self, codes):
        g, rnd, W = self.g, self.rnd, self.W

        def rvq(prefix, cols):
            total = None
            for i, c in enumerate(cols.T):
                e = W[f"{prefix}layers.{i}.codebook.embed_sum"][c] / np.maximum(
                    W[f"{prefix}layers.{i}.codebook.cluster_usage"][c], np.float32(1e-5))[:, None]
                e = rnd(e)
                total = e if total is None else rnd(total + e)
            return rnd.mm(total, W[prefix + "output_proj.weight"][:, :, 0])
        out = rvq("quantizer.semantic_residual_vector_quantizer.", codes[:, :g.n_semantic])
        if codes.shape[1] > g.n_semantic:
            out = rnd(out + rvq("quantizer.acoustic_residual_vector_quantizer.", codes[:, g.n_semantic:]))
        return out[:, :, None]                               # [B, hidden, 1]

    def _rope(self, x, cos, sin):
        """apply_rotary_pos_emb in the model dtype: each product and the sum are stored."""
        half = x.shape[-1] // 2
        rot = np.concatenate([-x[..., half:], x[..., :half]], -1)
        return self.rnd(self.rnd(x * cos) + self.rnd(rot * sin))

    def _transformer(self, h, slots):
        g, rnd, W = self.g, self.rnd, self.W
        B, T, _ = h.shape
        start = self.tokens[slots]
        positions = start[:, None] + np.arange(T)[None]
        ring_index = positions % g.ring
        self.key_pos[slots[:, None], ring_index] = positions
        key_pos = self.key_pos[slots][:, None, :]                       # [B, 1, R]
        qp = positions[:, :, None]
        mask = ((key_pos <= qp) & (key_pos > qp - g.window))[:, None]   # [B, 1, T, R]
        freqs = positions[:, :, None].astype(np.float32) * self.inv_freq[None, None, :]
        emb = np.concatenate([freqs, freqs], -1)
        cos = rnd(np.cos(emb).astype(np.float32))[:, None]             # [B, 1, T, hd]
        sin = rnd(np.sin(emb).astype(np.float32))[:, None]
        nh, hd = g.heads, g.head_dim
        for li in range(g.layers):
            p = f"decoder_transformer.layers.{li}."
            x = layer_norm(h, W[p + "input_layernorm.weight"], W[p + "input_layernorm.bias"], g.norm_eps, rnd)
            q = rnd.mm(x, W[p + "self_attn.q_proj.weight"]).reshape(B, T, nh, hd).transpose(0, 2, 1, 3)
            k = rnd.mm(x, W[p + "self_attn.k_proj.weight"]).reshape(B, T, nh, hd).transpose(0, 2, 1, 3)
            v = rnd.mm(x, W[p + "self_attn.v_proj.weight"]).reshape(B, T, nh, hd).transpose(0, 2, 1, 3)
            q, k = self._rope(q, cos, sin), self._rope(k, cos, sin)
            for t in range(T):
                self.kv[li, 0, slots, :, ring_index[:, t]] = k[:, :, t]
                self.kv[li, 1, slots, :, ring_index[:, t]] = v[:, :, t]
            K, V = self.kv[li, 0][slots], self.kv[li, 1][slots]            # [B, nh, R, hd]
            s = np.einsum("bhtd,bhrd->bhtr", q, K).astype(np.float32) * np.float32(hd ** -0.5)
            s = np.where(mask, s, np.float32(-np.inf))
            a = rnd(np.einsum("bhtr,bhrd->bhtd", softmax(s), V)).transpose(0, 2, 1, 3).reshape(B, T, nh * hd)
            a = rnd.mm(a, W[p + "self_attn.o_proj.weight"])
            h = rnd(h + rnd(W[p + "self_attn_layer_scale.scale"] * a))
            m = layer_norm(h, W[p + "post_attention_layernorm.weight"], W[p + "post_attention_layernorm.bias"],
                           g.norm_eps, rnd)
            m = rnd.mm(rnd(gelu(rnd.mm(m, W[p + "mlp.fc1.weight"]))), W[p + "mlp.fc2.weight"])
            h = rnd(h + rnd(W[p + "mlp_layer_scale.scale"] * m))
        self.tokens[slots] = start + T
        self.tokens[self.dummy] = 0
        return h

    def decode(self, slots, codes):
        """StaticMimi.decode/_forward (serve/fast_codec.py:186-192,247-277): codes [B, n_q] -> fp32 PCM
        [B, samples_per_frame] (pre-clamp)."""
        g, rnd, W = self.g, self.rnd, self.W
        slots = np.asarray(slots, np.int64)
        x = self._quantizer(np.asarray(codes, np.int64))
        x = self._convt(x, "upsample", slots, W["upsample.conv.weight"], None, g.upsample_stride, groups=g.hidden)
        x = self._transformer(x.transpose(0, 2, 1), slots).transpose(0, 2, 1)
        for idx, kind, cin, cout, k, stride in self.layout:
            p = f"decoder.layers.{idx}."
            key = f"decoder.{idx}"
            if kind == "conv":
                if idx > 0:
                    x = rnd(elu(x))
                x = self._conv(x, key, slots, W[p + "conv.weight"], W[p + "conv.bias"])
            elif kind == "convt":
                x = self._convt(rnd(elu(x)), key, slots, W[p + "conv.weight"], W[p + "conv.bias"], stride)
            else:
                r = self._conv(rnd(elu(x)), key + ".block.1", slots, W[p + "block.1.conv.weight"],
                               W[p + "block.1.conv.bias"])
                r = self._conv(rnd(elu(r)), key + ".block.3", slots, W[p + "block.3.conv.weight"],
                               W[p + "block.3.conv.bias"])
                x = rnd(x + r)
        return x[:, 0].astype(np.float32)
