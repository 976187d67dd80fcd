"""One engine tick on the CPU oracle -- TEST INFRASTRUCTURE (see oracle/__init__.py).

Composes the oracle stages the way Engine._tick does (maya3/engine.py:534-563): backbone step on each seat's
feedback vector, cb0 sampling with controlled stop, the depth loop, feedback write-back, the Mimi frame.  Used as
the checker of the tick-level parity tests and as the timed CPU baseline of bench.py.
"""
import numpy as np

from .backbone import BackboneOracle
from .depth import DepthOracle
from .mimi import MimiOracle
from .sampler import Cb0State, cb0_sample


class OracleTick:
    def __init__(self, weights, geom, max_slots, capacity, dtype="fp32", temp=0.7, top_k=64, greedy=False,
                 cb0_temp=0.9, cb0_top_k=64, cb0_rep=0.8, cb0_rep_win=12):
        self.g = geom
        self.greedy = greedy
        self.bb = BackboneOracle(weights, geom.backbone, max_slots, capacity, dtype)
        self.st = Cb0State(max_slots, temp=cb0_temp, top_k=cb0_top_k, rep=cb0_rep, rep_win=cb0_rep_win)
        self.depth = DepthOracle(weights, geom.depth, max_slots, dtype, temp=temp, top_k=top_k, greedy=greedy)
        self.mimi = MimiOracle(weights, geom.mimi, max_slots, dtype)
        self.feedback = np.zeros((max_slots + 1, geom.backbone.hidden), np.float32)
        self.rep = cb0_rep_win > 0 and cb0_rep > 0

    def cb0(self, h, slots):
        logits = self.bb.cb0_logits(h)
        if not self.greedy:
            return cb0_sample(logits, slots, self.st, self.rep, False) + (logits,)
        # greedy reference decode: argmax of the AEOS-removed distribution (maya3/engine.py:684-688)
        code = np.zeros(len(slots), np.int64)
        return code, np.argmax(logits[:, :2048], -1).astype(np.int64), logits

    def frame(self, slots, h):
        """Everything after the backbone: cb0, depth, feedback, Mimi.  Returns a dict of this frame's outputs."""
        slots = np.asarray(slots, np.int64)
        code, cb0, logits = self.cb0(h, slots)
        codes, fb = self.depth.step(slots, h, cb0)
        self.feedback[slots] = fb
        pcm = self.mimi.decode(slots, codes)
        return {"h": h, "cb0_logits": logits, "code": code, "codes": codes, "feedback": fb, "pcm": pcm,
                "depth_logits": self.depth.last_logits}

    def tick(self, slots):
        """A decode tick for seats already holding a prompt: the backbone input is each seat's feedback vector."""
        slots = np.asarray(slots, np.int64)
        h = self.bb.step(list(slots), self.feedback[slots])
        return self.frame(slots, h)
