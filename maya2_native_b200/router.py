"""Host-side stream router over engine replicas: one TickEngine per GPU, one process per GPU, no exchange between them.

Streams are independent, so the box scales by replication: a router in front assigns each new stream to one replica
and the stream stays there for its whole life (its KV cache, sampler and codec state live on that GPU).  The
reference serves one engine per process behind its HTTP/WS front (maya3/server.py:409-1060) and has no multi-replica
router; this module is the piece its configs[4] box measurement needs: Poisson arrivals routed round-robin (or to the
least-loaded replica) over the replicas.

Routing decisions are pure functions of the arrival index (round-robin) or of the replicas' reported loads
(least-loaded), so every process of a replicated job can derive its own share of a seeded global arrival stream
without talking to the others (``share``), which is how bench.py drives configs[4] under torchrun.
"""
from __future__ import annotations

import dataclasses

import numpy as np

POLICIES = ("round_robin", "least_loaded")


def poisson_arrivals(rate: float, duration: float, seed: int) -> np.ndarray:
    """Arrival times (seconds, ascending) of a Poisson process of `rate` arrivals per second on [0, duration)."""
    if rate < 0 or duration < 0:
        raise ValueError("rate and duration must be non-negative")
    if rate == 0 or duration == 0:
        return np.zeros(0)
    rng = np.random.default_rng(seed)
    n = int(rate * duration + 10 * np.sqrt(rate * duration) + 16)
    t = np.cumsum(rng.exponential(1.0 / rate, n))
    while t[-1] < duration:       # the bound above is exceeded with negligible probability; extend if it is not
        t = np.concatenate([t, t[-1] + np.cumsum(rng.exponential(1.0 / rate, n))])
    return t[t < duration]


@dataclasses.dataclass(frozen=True)
class Request:
    """One stream: arrival time (s), backbone prompt token ids, frame budget."""
    index: int
    t: float
    prompt: np.ndarray
    frames: int


def requests(arrivals: np.ndarray, vocab: int, indices=None, prompt=(20, 400), frames=(100, 1500),
             seed: int = 0) -> list:
    """The request behind each arrival (all of them, or those at `indices`): prompt length U[prompt], uniform random
    token ids, frame budget U[frames]; request i is drawn from its own generator (seed, i), so its content does not
    depend on which replica it is routed to."""
    out = []
    for i in (range(len(arrivals)) if indices is None else indices):
        i, t = int(i), arrivals[i]
        rng = np.random.default_rng((seed, i))
        P = int(rng.integers(prompt[0], prompt[1] + 1))
        T = int(rng.integers(frames[0], frames[1] + 1))
        out.append(Request(i, float(t), rng.integers(0, vocab, P), T))
    return out


class Router:
    """Assigns each new stream to one of `replicas` engines.

    round_robin   arrival k goes to replica (start + k) mod replicas;
    least_loaded  the replica with the fewest streams (active + queued) as reported in `loads`; ties go to the
                  first such replica after the last one chosen, so equal loads rotate like round-robin.
    """

    def __init__(self, replicas: int, policy: str = "round_robin", start: int = 0):
        if replicas < 1:
            raise ValueError("a router needs at least one replica")
        if policy not in POLICIES:
            raise ValueError(f"policy must be one of {POLICIES}, got {policy!r}")
        self.replicas = replicas
        self.policy = policy
        self._next = start % replicas
        self.routed = [0] * replicas

    def route(self, loads=None) -> int:
        if self.policy == "round_robin":
            r = self._next
        else:
            if loads is None or len(loads) != self.replicas:
                raise ValueError("least_loaded routing needs one load figure per replica")
            order = [(self._next + j) % self.replicas for j in range(self.replicas)]
            r = min(order, key=lambda i: loads[i])
        self._next = (r + 1) % self.replicas
        self.routed[r] += 1
        return r


def share(n_arrivals: int, rank: int, world: int) -> np.ndarray:
    """Indices of the arrivals that a round-robin router starting at replica 0 sends to replica `rank`."""
    if not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside [0, {world})")
    return np.arange(rank, n_arrivals, world)


__all__ = ["POLICIES", "Request", "Router", "poisson_arrivals", "requests", "share"]
