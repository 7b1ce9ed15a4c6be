"""Seeded sampler cases shared by the oracle pin test and the GPU test:
logit vectors with the shapes the references sample (32000 values), and
parameter sets spanning both samplers' branches (temperature 0 / greedy,
multinomial, top-p, repeat penalty above and below 1, out-of-range and
repeated history ids, ties at the top)."""
import numpy as np

VOCAB = 32000


def cases(n, seed=1, nonfinite=False):
    rng = np.random.default_rng(seed)
    out = []
    for c in range(n):
        x = rng.normal(0.0, 1.0 + 4.0 * rng.random(), VOCAB).astype(np.float32)
        if c % 5 == 0:  # ties at the top
            x[rng.integers(0, VOCAB, 40)] = x.max()
        if c % 7 == 3:  # a peaked distribution: few top-p candidates
            x[rng.integers(0, VOCAB, 3)] += 25.0
        if nonfinite and c % 4 == 1:
            x[rng.integers(0, VOCAB, 30)] = np.nan
            x[rng.integers(0, VOCAB, 10)] = -np.inf
        hist = rng.integers(-3, VOCAB + 3, int(rng.integers(0, 80))).astype(np.int32)
        if hist.size:
            hist = np.concatenate([hist, hist[: hist.size // 3]])  # repeated ids
        t = [0.0, 0.25, 0.7, 1.0, 1.6][c % 5]
        p = [0.0, 0.5, 0.9, 0.95, 1.0, -1.0, 0.99][c % 7]
        pen = [1.0, 1.1, 0.8, 1.3][c % 4]
        state = int(rng.integers(1, 2**63))
        out.append((x, hist, t, p, pen, state))
    return out
