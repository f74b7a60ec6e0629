"""The oracle's greedy choice (or_argmax) against the reference's loop, on the cases the device kernel must match:
Sampler.Sample at temperature 0 (src/Engine.cs:356-360) and Argmax (src/Engine.cs:329-334) both scan
best = 0; if (x[i] > x[best]) best = i, so ties keep the lower index, NaNs never win, a NaN at index 0 is never
replaced, and -0 equals +0."""
import numpy as np


def loop(v):
    best = 0
    for i in range(1, len(v)):
        if v[i] > v[best]:
            best = i
    return best


def test_oracle_argmax_follows_the_reference_loop(oracle):
    nan, inf = float("nan"), float("inf")
    cases = [
        [1.0], [2.0, 2.0], [1.0, 3.0, 3.0, 2.0], [nan, 5.0, 7.0], [1.0, nan, 7.0, nan], [nan, nan],
        [-0.0, 0.0, -1.0], [0.0, -0.0], [-inf, -inf, -inf], [-1.0, inf, inf], [-inf, nan, -3.0],
        [3.4e38, -3.4e38, 3.4e38], [1e-45, 0.0, 1e-45],
    ]
    rng = np.random.default_rng(0)
    for n in (5, 64, 1000):
        v = rng.integers(-3, 3, n).astype(np.float32)          # many ties
        cases.append(list(v))
    for c in cases:
        v = np.array(c, dtype=np.float32)
        assert oracle.argmax(v) == loop(v), c
