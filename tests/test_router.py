"""The host router of the replicated box: Poisson arrivals, per-arrival request content, round-robin and
least-loaded assignment, and each replica's own share of a seeded global arrival stream."""
import numpy as np
import pytest

from maya2_native_b200.router import Router, poisson_arrivals, requests, share


def test_poisson_arrivals_rate_and_order():
    t = poisson_arrivals(200.0, 50.0, seed=3)
    n = len(t)
    assert abs(n - 10000) < 5 * np.sqrt(10000)
    assert (np.diff(t) > 0).all() and t[0] >= 0 and t[-1] < 50.0
    gaps = np.diff(t)
    assert gaps.mean() == pytest.approx(1 / 200.0, rel=0.05)
    assert gaps.std() == pytest.approx(1 / 200.0, rel=0.05)        # exponential: std == mean
    assert np.array_equal(t, poisson_arrivals(200.0, 50.0, seed=3))
    assert len(poisson_arrivals(0.0, 5.0, seed=1)) == 0
    with pytest.raises(ValueError):
        poisson_arrivals(-1.0, 5.0, seed=1)


def test_request_content_does_not_depend_on_routing():
    t = poisson_arrivals(50.0, 2.0, seed=1)
    full = requests(t, 151936, prompt=(20, 400), frames=(100, 1500), seed=9)
    part = requests(t, 151936, indices=[7, 3], prompt=(20, 400), frames=(100, 1500), seed=9)
    assert [r.index for r in part] == [7, 3]
    for r in part:
        assert np.array_equal(r.prompt, full[r.index].prompt) and r.frames == full[r.index].frames
        assert r.t == t[r.index]
    assert all(20 <= len(r.prompt) <= 400 and 100 <= r.frames <= 1500 for r in full)
    assert all(0 <= int(r.prompt.min()) and int(r.prompt.max()) < 151936 for r in full)


def test_round_robin_matches_share():
    world, n = 3, 20
    rt = Router(world)
    got = [rt.route() for _ in range(n)]
    assert got == [i % world for i in range(n)]
    for r in range(world):
        assert list(share(n, r, world)) == [i for i in range(n) if got[i] == r]
    assert rt.routed == [7, 7, 6]
    with pytest.raises(ValueError):
        share(n, 3, 3)


def test_least_loaded():
    rt = Router(3, policy="least_loaded")
    assert rt.route([5, 2, 9]) == 1
    assert rt.route([1, 1, 1]) == 2          # tie: the first replica after the last one chosen
    assert rt.route([1, 1, 1]) == 0
    assert rt.route([0, 4, 0]) == 2
    with pytest.raises(ValueError):
        rt.route()
    with pytest.raises(ValueError):
        Router(2, policy="random")
    with pytest.raises(ValueError):
        Router(0)
