"""FastDepth: drop-in replacement of serve/fast_depth.py:FastDepth on the B200 C ABI.

Same constructor arguments, ``set_speaker``/``warmup``/``bucket_for``/``__call__`` and engine-written attributes
(``row_seed``, ``row_ctr``).  Sampling always uses the per-slot Philox streams of the fused path (``fused=True``
in the engine); ``compile``/``fused`` are accepted for signature compatibility.  One ``m3_depth_step`` per call,
replayed from a CUDA graph per batch bucket (serve/fast_depth.py:205-227).
"""
from __future__ import annotations

import sys
from collections.abc import Mapping

import torch

from . import _lib as L
from .config import DepthGeom


def _named(model) -> Mapping:
    if isinstance(model, Mapping):
        return model
    sd = {"depth." + k: v for k, v in model.depth.state_dict().items()}
    sd.update({"audio_in." + k: v for k, v in model.audio_in.state_dict().items()})
    return sd


class FastDepth:
    def __init__(self, model, max_slots, dtype=torch.bfloat16, temp=0.7, top_k=64,
                 batch_buckets=(1, 2, 4, 8, 16, 24, 32, 48, 64, 80, 96), seed=1234, greedy=False, compile=False,
                 fused=False, geom: DepthGeom | None = None, device=None):
        if dtype not in (torch.bfloat16, "bf16"):
            raise ValueError("this build serves the depth stack in bf16 only")
        sd = _named(model)
        if geom is None:
            # the reference keeps the depth head count and the level -> weight-group map as globals of the module
            # that defines DepthV2 (tts/model/depth_v2.py:45-47), which its own FastDepth imports
            d = model.depth
            mod = sys.modules.get(type(d).__module__)
            gol = tuple(getattr(mod, "GROUP_OF_LEVEL", ())[:d.n_q])
            geom = DepthGeom(layers=len(d.groups[0]), d=d.in_proj.out_features, heads=int(getattr(mod, "H", 8)),
                             ffn=d.groups[0][0].f1.out_features, n_q=d.n_q, n_codes=d.n_codes,
                             rank=d.code_up.in_features, d_backbone=d.in_proj.in_features, group_of_level=gol)
        self.geom = g = geom
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.dtype = torch.bfloat16
        self.max_slots = int(max_slots)
        self.temp, self.top_k, self.greedy = float(temp), int(top_k), bool(greedy)
        self.batch_buckets = tuple(sorted(set(int(b) for b in batch_buckets)))
        self.n_codes = g.n_codes
        dev, bf = self.device, self.dtype

        def w(name):
            return sd[name].detach().to(dev, bf).contiguous()
        with torch.inference_mode():
            NL, D = g.n_q, g.d
            self.in_proj = w("depth.in_proj.weight")
            code_lo, code_up = w("depth.code_lo.weight"), w("depth.code_up.weight")
            table = torch.empty(code_lo.shape[0], D, dtype=bf, device=dev)
            L.check(L.load().m3_gemm_bf16(code_lo.data_ptr(), code_lo.shape[1], code_up.data_ptr(), code_up.shape[1],
                                          table.data_ptr(), D, code_lo.shape[0], D, code_lo.shape[1], 0,
                                          L.stream_ptr()), "prefix table")
            lvl = w("depth.level_emb.weight")
            # position k+1 of the prefix = code_up(code_lo[cb_k + k*n_codes]) + level_emb[k+1] (fast_depth.py:48-50)
            self.embed = (table.view(NL - 1, g.n_codes, D) + lvl[1:NL, None]).contiguous()
            self.level0 = lvl[0].clone()
            self._w = {k: [] for k in ("n1_w", "n1_b", "n2_w", "n2_b", "qkv", "o", "f1", "f2")}
            for grp in range(g.n_groups):
                for li in range(g.layers):
                    p = f"depth.groups.{grp}.{li}."
                    for key, name in (("n1_w", "n1.weight"), ("n1_b", "n1.bias"), ("n2_w", "n2.weight"),
                                      ("n2_b", "n2.bias"), ("qkv", "qkv.weight"), ("o", "o.weight"),
                                      ("f1", "f1.weight"), ("f2", "f2.weight")):
                        self._w[key].append(w(p + name))
            self.norm_w, self.norm_b = w("depth.norm.weight"), w("depth.norm.bias")
            self.heads = [w(f"depth.heads.{i}.weight") for i in range(NL - 1)]
            self.cross_kv = [w(f"depth.cross.{i}.kv.weight") for i in range(g.layers)]
            self.cross_o = [w(f"depth.cross.{i}.o.weight") for i in range(g.layers)]
            self.audio_table = w("audio_in.table.weight")
            self.audio_norm = w("audio_in.norm.weight")
            self.cross_const = torch.zeros(self.max_slots + 1, g.layers, D, device=dev, dtype=bf)
        self.generator = torch.Generator(device=dev).manual_seed(int(seed))
        self.seed_t = torch.full((1,), int(seed) % (2 ** 31 - 1), device=dev, dtype=torch.int32)
        self.row_seed = torch.zeros(self.max_slots + 1, device=dev, dtype=torch.int32)
        self.row_ctr = torch.zeros(self.max_slots + 1, device=dev, dtype=torch.int32)
        self.per_row = True
        self.fused = True
        self.pool = None
        self.graphs = {}
        self._handle = self._create()

    def _create(self):
        g = self.geom
        gol = (L.i32 * 64)(*([0] + [int(x) for x in g.group_of_level[1:]] + [0] * (64 - g.n_q)))
        cfg = L.DepthConfig(g.layers, g.d, g.heads, g.ffn, g.n_q, g.n_codes, g.d_backbone, g.n_groups, gol,
                            self.max_slots, max(self.batch_buckets), g.ln_eps, float(1.0 / self.temp), self.top_k,
                            int(self.greedy))
        arr = {k: L.ptr_array([t.data_ptr() for t in v]) for k, v in self._w.items()}
        heads = L.ptr_array([t.data_ptr() for t in self.heads])
        ckv = L.ptr_array([t.data_ptr() for t in self.cross_kv])
        co = L.ptr_array([t.data_ptr() for t in self.cross_o])
        self._keep = (arr, heads, ckv, co)
        wts = L.DepthWeights(self.in_proj.data_ptr(), self.embed.data_ptr(), self.level0.data_ptr(), arr["n1_w"],
                             arr["n1_b"], arr["n2_w"], arr["n2_b"], arr["qkv"], arr["o"], arr["f1"], arr["f2"],
                             self.norm_w.data_ptr(), self.norm_b.data_ptr(), heads, ckv, co,
                             self.audio_table.data_ptr(), self.audio_norm.data_ptr(), self.cross_const.data_ptr(),
                             self.row_seed.data_ptr(), self.row_ctr.data_ptr())
        h = L.vp()
        L.check(L.load().m3_depth_create(cfg, wts, h), "m3_depth_create")
        return h

    def debug_logits(self):
        """Keep every level's head logits (bf16 [n_q - 1, max_rows, n_codes]) from the next step on (steps captured
        into graphs afterwards included); returns the buffer, whose rows [:B] hold the latest step's seats."""
        g = self.geom
        buf = torch.zeros(g.n_q - 1, max(self.batch_buckets), g.n_codes, device=self.device, dtype=torch.bfloat16)
        L.check(L.load().m3_depth_debug_logits(self._handle, buf.data_ptr(), buf.numel() * 2),
                "m3_depth_debug_logits")
        self._dbg = buf
        return buf

    def close(self):
        if getattr(self, "_handle", None):
            self.graphs.clear()
            L.load().m3_depth_destroy(self._handle)
            self._handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def device_status(self, clear=True) -> int:
        s = L.i32(0)
        L.check(L.load().m3_depth_status(self._handle, s, int(clear)), "m3_depth_status")
        return int(s.value)

    @torch.inference_mode()
    def set_speaker(self, slot, mem, ref_mask):
        """serve/fast_depth.py:72-82: one reference token per slot -> per-layer constant o(v(mem))."""
        if mem.ndim != 3 or mem.shape[0] != 1 or mem.shape[1] != 1 or tuple(ref_mask.shape) != (1, 1):
            raise ValueError(f"FastDepth serves exactly one reference per slot; got mem {tuple(mem.shape)}")
        if not 0 <= slot < self.max_slots:
            raise IndexError(f"slot {slot} outside 0..{self.max_slots - 1}")
        m = mem.reshape(-1).to(self.device, self.dtype).contiguous()
        keep = float(bool(ref_mask.reshape(-1)[0]))
        L.check(L.load().m3_depth_set_speaker(self._handle, int(slot), m.data_ptr(), keep, L.stream_ptr()),
                "m3_depth_set_speaker")

    def _launch(self, s, stream=None):
        L.check(L.load().m3_depth_step(self._handle, s["slots_idx"].data_ptr(), s["h"].data_ptr(),
                                       s["cb0"].data_ptr(), s["codes"].data_ptr(), s["feedback"].data_ptr(),
                                       s["slots_idx"].shape[0], L.stream_ptr(stream)), "m3_depth_step")

    @torch.inference_mode()
    def _capture(self, bucket):
        if bucket in self.graphs:
            return self.graphs[bucket]
        dev, g = self.device, self.geom
        s = {"slots_idx": torch.full((bucket,), self.max_slots, device=dev, dtype=torch.long),
             "h": torch.zeros(bucket, g.d_backbone, device=dev, dtype=self.dtype),
             "cb0": torch.zeros(bucket, device=dev, dtype=torch.long),
             "codes": torch.zeros(bucket, g.n_q, device=dev, dtype=torch.long),
             "feedback": torch.zeros(bucket, g.d_backbone, device=dev, dtype=self.dtype),
             "last_slots": None}
        stream = torch.cuda.Stream()
        stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(stream):
            for _ in range(2):
                self._launch(s, stream)
        torch.cuda.current_stream().wait_stream(stream)
        self.row_ctr[self.max_slots] = 0
        if self.pool is None:
            self.pool = torch.cuda.graph_pool_handle()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, pool=self.pool, stream=stream):
            self._launch(s, stream)
        s["graph"] = graph
        self.graphs[bucket] = s
        return s

    def warmup(self, batch_buckets=None):
        for bucket in sorted(set(batch_buckets or self.batch_buckets), reverse=True):
            self._capture(int(bucket))

    def bucket_for(self, batch):
        for bucket in self.batch_buckets:
            if bucket >= batch:
                return bucket
        raise ValueError(f"batch {batch} exceeds the largest bucket {self.batch_buckets[-1]}")

    @torch.inference_mode()
    def __call__(self, slots, h, cb0):
        """serve/fast_depth.py:240-257 -> (codes [B, n_q] long, feedback [B, d_backbone]) owned copies."""
        B = len(slots)
        if h.shape[0] != B or cb0.shape[0] != B:
            raise ValueError("slots, h and cb0 must have the same batch size")
        s = self._capture(self.bucket_for(B))
        key = tuple(slots)
        if key != s["last_slots"]:
            if any(not 0 <= slot < self.max_slots for slot in key):
                raise IndexError(f"slot outside 0..{self.max_slots - 1}")
            padded = list(key) + [self.max_slots] * (s["slots_idx"].shape[0] - B)
            s["slots_idx"].copy_(torch.tensor(padded, dtype=torch.long))
            s["last_slots"] = key
        s["h"][:B].copy_(h)
        s["cb0"][:B].copy_(cb0)
        s["graph"].replay()
        return s["codes"][:B].clone(), s["feedback"][:B].clone()
