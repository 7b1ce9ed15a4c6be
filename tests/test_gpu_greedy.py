"""Greedy steps on the device (embedding lookup + argmax in the token kernel)
against the logits path with the host argmax of decode_host.cpp:703-717:
ids and logits bit-exact; the device argmax on its edge cases."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

LAYERS, SEED, STEPS = 2, 11, 10


def host_argmax(logits, n=32000):
    """First index of the maximum of logits[:n], NaN skipped (-1 if none)."""
    best, idx = None, -1
    for i in range(n):
        v = float(logits[i])
        if v != v:
            continue
        if best is None or v > best:
            best, idx = v, i
    return idx


@pytest.fixture(scope="module")
def greedy_model(synth):
    return synth.model_banks(LAYERS, SEED), synth.embeddings(SEED)


def test_greedy_matches_logits_path(pkg, rope_lut, greedy_model):
    banks, emb = greedy_model
    with pkg.Context(num_layers=LAYERS, kv_capacity=64) as g, pkg.Context(num_layers=LAYERS, kv_capacity=64) as r:
        for c in (g, r):
            c.load_banks(banks)
            c.load_rope(rope_lut)
        g.load_embeddings(emb)
        tok = 1
        for pos in range(STEPS):
            nxt, logits = g.decode_greedy(pos, tok, want_logits=True)
            ref = r.decode_token(pos, emb[tok * 4096:(tok + 1) * 4096])
            assert np.array_equal(logits.view(np.uint32), ref.view(np.uint32)), pos
            assert nxt == host_argmax(ref), pos
            tok = nxt


def test_device_argmax_edge_cases(pkg):
    ctx = pkg.Context(num_layers=1, kv_capacity=16)
    rng = np.random.default_rng(5)
    cases = []
    x = rng.normal(size=32256).astype(np.float32)
    cases.append(x)
    y = x.copy()
    y[[100, 200, 31999]] = 50.0  # ties: the first wins
    cases.append(y)
    z = x.copy()
    z[7] = np.nan
    z[8] = 60.0
    z[9] = np.nan
    cases.append(z)
    w = np.full(32256, -1.0, np.float32)
    w[300] = -0.0
    w[299] = 0.0  # +0 and -0 are equal: the first (299) wins
    cases.append(w)
    w2 = w.copy()
    w2[299], w2[300] = -0.0, 0.0
    cases.append(w2)
    p = np.full(32256, -3.0, np.float32)
    p[32100] = 10.0  # padding rows beyond 32000 never count
    cases.append(p)
    nan = np.full(32256, np.nan, np.float32)
    cases.append(nan)
    for i, c in enumerate(cases):
        assert ctx.argmax(c[:32000]) == host_argmax(c), i
    short = x[:1000].copy()
    assert ctx.argmax(short) == host_argmax(short, n=1000)
    ctx.close()
