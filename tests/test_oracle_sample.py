"""The oracle's Sampler.Sample (or_sample) against the reference's method restated as a Python loop, and the
reference's own sampler test (tests/Tests.cs:555-566, SamplerWorks) with the generator's draws passed in.

Sampler.Sample (src/Engine.cs:361-380): greedy at temperature <= 0; else p[i] = exp((x[i] - max) / temperature)
in double with the difference taken in float; top_p >= 1 walks r = draw * sum down the ids in index order; top_p < 1
sorts by p descending, keeps the first k whose running sum reaches top_p * sum, and walks pick = draw * cum down
those k. The draw is rng.NextDouble(), taken once per call at temperature > 0."""
import math

import numpy as np
import pytest


def py_sample(x, temperature, top_p, draw):
    """Sampler.Sample with the draw passed in, one term at a time (equal probabilities in ascending id order)."""
    x = np.asarray(x, dtype=np.float32)
    n = x.size
    best = 0
    for i in range(1, n):
        if x[i] > x[best]:
            best = i
    if temperature <= 0:
        return best
    mx = x[best]
    p = [math.exp(float(np.float32(x[i] - mx)) / temperature) for i in range(n)]
    s = 0.0
    for v in p:
        s += v
    if top_p >= 1.0:
        r = draw * s
        for i in range(n):
            r -= p[i]
            if r <= 0:
                return i
        return best
    idx = sorted(range(n), key=lambda i: (-p[i], i))
    cum, limit, k = 0.0, top_p * s, 0
    while k < n:
        cum += p[idx[k]]
        k += 1
        if cum >= limit:
            break
    pick = draw * cum
    for i in range(k):
        pick -= p[idx[i]]
        if pick <= 0:
            return idx[i]
    return idx[0]


def test_sampler_works_with_passed_draws(oracle):
    """SamplerWorks: greedy gives 1; one generator state gives one id; at top_p 0.5 only the two large logits are
    ever chosen (here over a grid of draws in [0, 1), the values rng.NextDouble() can return)."""
    logits = np.array([0.1, 3.0, 0.2, 2.9], dtype=np.float32)
    assert oracle.sample(logits, 0, 1, 0.5)[0] == 1
    assert oracle.sample(logits, 1, 1, 0.37)[0] == oracle.sample(logits, 1, 1, 0.37)[0]
    for d in np.linspace(0.0, 1.0, 201, endpoint=False):
        k = oracle.sample(logits, 1, 0.5, float(d))[0]
        assert k in (1, 3), (d, k)
    # top_p 1: every id is reachable, in index order of the cumulative probabilities
    seen = {oracle.sample(logits, 1, 1, float(d))[0] for d in np.linspace(0.0, 1.0, 2001, endpoint=False)}
    assert seen == {0, 1, 2, 3}


@pytest.mark.parametrize("n", [1, 2, 5, 37, 300])
def test_oracle_sample_follows_the_reference_loop(oracle, n):
    rng = np.random.default_rng(n)
    for case in range(60):
        if case % 3 == 0:
            x = rng.integers(-4, 4, n).astype(np.float32)           # many equal probabilities
        else:
            x = (rng.standard_normal(n) * rng.uniform(0.5, 8)).astype(np.float32)
        t = float(rng.choice([0.0, -1.0, 0.05, 0.4, 1.0, 2.5]))
        p = float(rng.choice([1.0, 1.5, 0.95, 0.5, 0.1, 0.0]))
        d = float(rng.random())
        assert oracle.sample(x, t, p, d)[0] == py_sample(x, t, p, d), (n, case, t, p, d)


def test_oracle_sample_edges(oracle):
    x = np.array([0.0, 0.0, 0.0, 0.0], dtype=np.float32)
    # equal probabilities: index order at top_p 1, ascending ids in the nucleus
    assert [oracle.sample(x, 1, 1, d)[0] for d in (0.0, 0.2, 0.3, 0.6, 0.99)] == [0, 0, 1, 2, 3]
    assert [oracle.sample(x, 1, 0.5, d)[0] for d in (0.0, 0.4, 0.6, 0.99)] == [0, 0, 1, 1]
    # draw 0 takes the first id with a positive probability (r - p <= 0 at once)
    assert oracle.sample(np.array([-1e4, 1.0, 2.0], dtype=np.float32), 1, 1, 0.0)[0] == 0
    # top_p 0 keeps the most probable id alone
    y = np.array([0.5, 2.0, 1.9, -3.0], dtype=np.float32)
    assert {oracle.sample(y, 1, 0.0, d)[0] for d in (0.0, 0.5, 0.999)} == {1}
    # a tiny temperature underflows every other probability to zero: the greedy id
    assert oracle.sample(y, 1e-3, 1.0, 0.999)[0] == 1
    # the margin is the relative distance of the draw from the nearest boundary
    i, m = oracle.sample(x, 1, 1, 0.3)
    assert i == 1 and abs(m - 0.05) < 1e-12
