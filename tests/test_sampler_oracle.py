"""The oracle's restatement of the samplers (oracle/i4d_oracle.c, i4o_sample)
pinned against the reference emulator's own sampler compiled from its source
(emulator:1411-1569 through oracle/_ref): same token and same advanced RNG
state on every seeded case.  The host sampler (decode_host.cpp:724-868) needs
the XRT runtime to compile; its restatement shares the pinned pieces (RNG,
serial sums, walks) and is checked here on its own branches."""
import numpy as np
import pytest

import sampler_cases


def test_emulator_sampler_pinned(oracle):
    import oracle as orc
    if not orc.ref_available():
        pytest.skip("reference emulator not built here")
    ref = orc.RefEmulator()
    for i, (x, hist, t, p, pen, st) in enumerate(sampler_cases.cases(150)):
        a = oracle.sample(1, x, hist, t, p, pen, st)
        b = ref.sample(x, hist, t, p, pen, st)
        assert a == b, (i, t, p, pen, a, b)


def host_argmax(x):
    v = np.where(np.isnan(x), -np.inf, x)
    ok = ~np.isnan(x)
    if not ok.any():
        return -1
    return int(np.flatnonzero(ok & (v == v[ok].max()))[0])


def test_host_sampler_branches(oracle):
    rng = np.random.default_rng(3)
    x = rng.normal(0, 2, 32000).astype(np.float32)
    # temperature 0, no penalty: argmax with NaN skipped; no coin drawn
    y = x.copy()
    y[:5] = np.nan
    t, st = oracle.sample(0, y, np.zeros(0, np.int32), 0.0, 0.9, 1.0, 7)
    assert t == host_argmax(y) and st == 7
    # every logit NaN: the host's exception
    t, _ = oracle.sample(0, np.full(32000, np.nan, np.float32), np.zeros(0, np.int32), 0.0, 0.0, 1.0, 7)
    assert t == -1
    t, _ = oracle.sample(0, np.full(32000, np.inf, np.float32), np.zeros(0, np.int32), 0.8, 0.0, 1.0, 7)
    assert t == -2
    # the repeat penalty is applied once per distinct id: a repeated id equals a single one
    h1 = np.array([5, 5, 5, 9], np.int32)
    h2 = np.array([5, 9], np.int32)
    assert oracle.sample(0, x, h1, 0.0, 0.0, 1.3, 1) == oracle.sample(0, x, h2, 0.0, 0.0, 1.3, 1)
    # a draw advances the state exactly as xorshift64*; same state -> same token
    a = oracle.sample(0, x, h2, 0.9, 0.9, 1.1, 12345)
    b = oracle.sample(0, x, h2, 0.9, 0.9, 1.1, 12345)
    assert a == b and a[1] != 12345
    s = 12345
    s ^= s >> 12
    s ^= (s << 25) & (2**64 - 1)
    s ^= s >> 27
    assert a[1] == s
