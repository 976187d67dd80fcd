"""Cb0Sampler: the engine's cb0 sampling + controlled stop (maya3/engine.py:652-694) on the B200 C ABI.

The per-slot state tensors carry the engine's names (``frames_t``, ``min_t``, ``hazard_t``, ``aeos_bias``,
``temp_t``, ``topk_t``, ``topp_t``, ``rep_t``, ``seed_t``, ``ctr_t``, ``hist_t``; maya3/engine.py:210-223) so the
engine's admission code (``_bind``, maya3/engine.py:420-447) writes them unchanged.  One call runs the cb0 head
GEMM and one fused sampler kernel per row.
"""
from __future__ import annotations

import torch

from . import _lib as L
from .config import AEOS_CLASS, N_CODES


class Cb0Sampler:
    def __init__(self, head_weight, max_slots, max_rows=None, temp=0.9, top_k=64, top_p=1.0, rep=0.8, rep_win=12,
                 device=None):
        dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.device = dev
        m = int(max_slots) + 1
        self.max_slots = int(max_slots)
        self.max_rows = int(max_rows or max_slots)
        self.rep_win = int(rep_win)
        self.cfg_rep = float(rep)
        self.head = head_weight.detach().to(dev, torch.bfloat16).contiguous()
        self.n_cls, self.hidden = self.head.shape
        if self.n_cls != N_CODES + 1:
            raise ValueError(f"cb0 head must have {N_CODES + 1} classes, got {self.n_cls}")
        self.frames_t = torch.zeros(m, device=dev, dtype=torch.long)
        self.min_t = torch.zeros(m, device=dev, dtype=torch.long)
        self.hazard_t = torch.zeros(m, device=dev, dtype=torch.float32)
        self.aeos_bias = torch.zeros(m, device=dev, dtype=torch.float32)
        self.temp_t = torch.full((m,), float(temp), device=dev, dtype=torch.float32)
        self.topk_t = torch.full((m,), int(top_k), device=dev, dtype=torch.long)
        self.topp_t = torch.full((m,), float(top_p), device=dev, dtype=torch.float32)
        self.rep_t = torch.full((m,), float(rep), device=dev, dtype=torch.float32)
        self.seed_t = torch.zeros(m, device=dev, dtype=torch.int32)
        self.ctr_t = torch.zeros(m, device=dev, dtype=torch.int32)
        self.hist_t = torch.full((m, max(1, self.rep_win)), -1, device=dev, dtype=torch.long)
        self.any_rep = False
        self.any_top_p = float(top_p) < 1.0
        lib = L.load()
        cfg = L.Cb0Config(self.hidden, self.n_cls, self.max_slots, self.max_rows, self.rep_win)
        st = L.Cb0State(*[t.data_ptr() for t in (self.head, self.frames_t, self.min_t, self.hazard_t, self.aeos_bias,
                                                 self.temp_t, self.topk_t, self.topp_t, self.rep_t, self.seed_t,
                                                 self.ctr_t, self.hist_t)])
        h = L.vp()
        L.check(lib.m3_cb0_create(cfg, st, h), "m3_cb0_create")
        self._handle = h

    def close(self):
        if getattr(self, "_handle", None):
            L.load().m3_cb0_destroy(self._handle)
            self._handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def device_status(self, clear=True) -> int:
        """The handle's device status word (M3_DEV_BAD_SLOT after a row named a slot outside [0, max_slots]);
        synchronises with the device."""
        s = L.i32(0)
        L.check(L.load().m3_cb0_status(self._handle, s, int(clear)), "m3_cb0_status")
        return int(s.value)

    def copy_logits(self, rows):
        """The bf16 head logits [rows, 2049] the last step's sampler read (a copy, stream-ordered)."""
        out = torch.empty(int(rows), self.n_cls, device=self.device, dtype=torch.bfloat16)
        L.check(L.load().m3_cb0_copy_logits(self._handle, out.data_ptr(), int(rows), L.stream_ptr()),
                "m3_cb0_copy_logits")
        return out

    def flags(self):
        """The engine's host-side switches: penalty when cb0_rep_win > 0 and (cb0_rep > 0 or any request set one);
        top-p when any request asked for top_p < 1 (maya3/engine.py:660,669)."""
        return int(self.rep_win > 0 and (self.cfg_rep > 0 or self.any_rep)), int(self.any_top_p)

    @torch.inference_mode()
    def __call__(self, h, idx, out=None):
        """h [B, hidden] bf16 (device), idx [B] long slots -> (stop code [B], cb0 [B]) long."""
        B = int(idx.shape[0])
        if h.shape[0] != B:
            raise ValueError("h and idx must have the same batch size")
        if B > self.max_rows:
            raise ValueError(f"batch {B} exceeds max_rows {self.max_rows}")
        h = h.to(torch.bfloat16).contiguous()
        idx = idx.to(self.device, torch.long).contiguous()
        code, cb0 = out if out is not None else (torch.empty(B, dtype=torch.long, device=self.device),
                                                 torch.empty(B, dtype=torch.long, device=self.device))
        rep, top_p = self.flags()
        L.check(L.load().m3_cb0_step(self._handle, h.data_ptr(), idx.data_ptr(), code.data_ptr(), cb0.data_ptr(), B,
                                     rep, top_p, L.stream_ptr()), "m3_cb0_step")
        return code, cb0

    @torch.inference_mode()
    def sample_logits(self, logits, idx, apply_rep=None, apply_top_p=None):
        """The sampler alone on fp32 logits [B, 2049]."""
        B = int(idx.shape[0])
        logits = logits.to(self.device, torch.float32).contiguous()
        idx = idx.to(self.device, torch.long).contiguous()
        code = torch.empty(B, dtype=torch.long, device=self.device)
        cb0 = torch.empty(B, dtype=torch.long, device=self.device)
        rep, top_p = self.flags()
        rep = rep if apply_rep is None else int(apply_rep)
        top_p = top_p if apply_top_p is None else int(apply_top_p)
        L.check(L.load().m3_cb0_sample_logits(self._handle, logits.data_ptr(), idx.data_ptr(), code.data_ptr(),
                                              cb0.data_ptr(), B, rep, top_p, L.stream_ptr()), "m3_cb0_sample_logits")
        return code, cb0


def topk_sample(logits, seeds, ctrs, level, temp, top_k, greedy=False):
    """serve/fast_depth_kernels.py:topk_sample on the C ABI: logits [B, V] (bf16 or fp32), per-row seed/counter."""
    B, V = logits.shape
    bf = logits.dtype == torch.bfloat16
    logits = logits.contiguous() if bf else logits.float().contiguous()
    out = torch.empty(B, dtype=torch.long, device=logits.device)
    seeds = seeds.to(logits.device, torch.int32).contiguous()
    ctrs = ctrs.to(logits.device, torch.int32).contiguous()
    L.check(L.load().m3_topk_sample(logits.data_ptr(), int(bf), B, V, seeds.data_ptr(), ctrs.data_ptr(), int(level),
                                    float(1.0 / temp), int(top_k), int(greedy), out.data_ptr(), L.stream_ptr()),
            "m3_topk_sample")
    return out


__all__ = ["Cb0Sampler", "topk_sample", "AEOS_CLASS"]
