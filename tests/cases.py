"""Small structural test cases for the PLE path.

The categories mirror the reference test fixtures (``tests/utils/
generate_bins.py``: equal, ragged, single_bin, all_single_bin;
``tests/utils/generate_input.py``: samples inside, below and above the edge
range) with edge values of this project's own choosing, plus cases the
reference does not have: exact edge ties, +-inf inputs, wide quantile bins.
"""
from __future__ import annotations

import numpy as np

BIN_CASES = ("equal", "ragged", "single_bin", "all_single_bin", "ties", "wide")


def make_bins(case: str) -> list[np.ndarray]:
    f32 = lambda v: np.asarray(v, dtype=np.float32)  # noqa: E731
    if case == "equal":            # 3 features x 4 bins
        return [f32([-3.5, -1.25, 0.0, 2.0, 4.5]),
                f32([-2.0, -0.5, 1.0, 2.5, 7.0]),
                f32([-6.0, -3.0, -0.25, 1.75, 6.0])]
    if case == "ragged":           # 4, 2, 5, 3 bins
        return [f32([-3.5, -1.25, 0.0, 2.0, 4.5]),
                f32([-2.5, 0.5, 3.0]),
                f32([-5.0, -2.75, -1.5, 0.25, 2.0, 6.5]),
                f32([-1.5, 1.25, 4.0, 8.5])]
    if case == "single_bin":       # mixes 1-bin and multi-bin features
        return [f32([-3.5, -1.25, 0.0, 2.0, 4.5]),
                f32([-0.75, 2.5]),
                f32([-4.5, -0.5, 1.5, 5.5])]
    if case == "all_single_bin":
        return [f32([-2.5, 1.5]), f32([-1.25, 3.75]), f32([-4.0, 4.0])]
    if case == "ties":             # integer edges: inputs hit interior edges exactly
        return [f32([0, 1, 2, 3, 5, 8]), f32([-2, 0, 2, 4]), f32([1, 2]), f32([0, 3, 4, 5, 6, 7, 8, 9, 12])]
    if case == "wide":             # 64 quantile bins for a few features
        rng = np.random.default_rng(99)
        return [np.quantile(rng.standard_normal(20_000), np.linspace(0, 1, 65)).astype(np.float32)
                for _ in range(5)]
    raise ValueError(case)


def sample_x(bins, n: int, seed: int, *, integer: bool = False, specials: bool = False) -> np.ndarray:
    """Seeded ``[n, F]`` inputs: half spread around the edge range, a quarter
    below the first edge, a quarter above the last (every region of the
    encoding, including both unbounded end bins).  ``integer`` rounds to
    integers (exact edge ties for integer edges); ``specials`` plants exact
    edge values and +-inf."""
    assert n % 4 == 0
    rng = np.random.default_rng(seed)
    cols = []
    for e in bins:
        lo, hi = float(e[0]), float(e[-1])
        span = hi - lo
        inside = rng.standard_normal(n // 2) * span / 2 + (lo + hi) / 2
        below = lo - rng.random(n // 4) * span
        above = hi + rng.random(n // 4) * span
        c = np.concatenate([inside, below, above])
        rng.shuffle(c)
        if integer:
            c = np.round(c)
        if specials:
            m = min(len(e), n // 4)
            c[:m] = e[:m]
            c[m] = np.inf
            c[m + 1] = -np.inf
        cols.append(c.astype(np.float32))
    return np.stack(cols, axis=1)


def init_params(f: int, b: int, d: int, version: str, seed: int):
    """Parameter init of the reference correctness tests
    (``tests/test_correctness.py:45-76``): W ~ U(0.05, 0.25),
    bias ~ U(0.10, 0.30), w0 ~ U(-0.2, 0.2), b0 ~ U(-0.1, 0.1)."""
    rng = np.random.default_rng(seed)
    w = rng.uniform(0.05, 0.25, size=(f, b, d)).astype(np.float32)
    if version == "A":
        return w, rng.uniform(0.10, 0.30, size=(f, d)).astype(np.float32), None, None
    return (w, None, rng.uniform(-0.2, 0.2, size=(f, d)).astype(np.float32),
            rng.uniform(-0.1, 0.1, size=(f, d)).astype(np.float32))
