"""CPU oracle for the Maya3 decode tick -- TEST INFRASTRUCTURE, not product code.

A numpy restatement of the reference's per-tick algorithm (backbone decode over the static per-seat KV cache, the
cb0 sampler with controlled stop, the depth RVQ level loop with top-k sampling, and the one-frame Mimi decoder).
Each function cites the reference file:line it follows.  It is pinned against fixtures produced by the reference
itself (tests/golden/make_golden.py).

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference arm may import this package, and only
as the checker or the timed CPU baseline: the CUDA product path never calls into it.
"""
