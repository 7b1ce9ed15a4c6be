"""The device sampler (i4d_sample, i4d_decode_sample) against the oracle's
restatement of both reference samplers (decode_host.cpp:724-868 and
emulator:1411-1569, the latter pinned against the compiled emulator in
test_sampler_oracle.py): token and advanced RNG state identical on every
seeded case, over consecutive draws with one sampler state."""
import numpy as np
import pytest

import sampler_cases

pytestmark = pytest.mark.gpu

LAYERS, SEED = 2, 11


@pytest.fixture(scope="module")
def ctx(pkg):
    with pkg.Context(num_layers=1, kv_capacity=8) as c:
        yield c


def _dev(x):
    import torch
    return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).cuda()


@pytest.mark.parametrize("mode", [0, 1])
def test_sample_matches_oracle(pkg, ctx, oracle, mode):
    for i, (x, hist, t, p, pen, st) in enumerate(sampler_cases.cases(60, seed=5 + mode, nonfinite=(mode == 0))):
        d = _dev(x)
        s = pkg.Sampler(temperature=t, top_p=p, repeat_penalty=pen, mode=mode, rng_state=st)
        want, want_st = oracle.sample(mode, x, hist, t, p, pen, st)
        if want < 0:
            with pytest.raises(pkg.I4DError):
                ctx.sample(d.data_ptr(), hist, s)
            continue
        got = ctx.sample(d.data_ptr(), hist, s)
        assert (got, s.rng_state) == (want, want_st), (i, t, p, pen)
        # a second draw from the advanced state
        want2, want_st2 = oracle.sample(mode, x, hist, t, p, pen, want_st)
        got2 = ctx.sample(d.data_ptr(), hist, s)
        assert (got2, s.rng_state) == (want2, want_st2), (i, "second draw")


def test_sample_edge_cases(pkg, ctx, oracle):
    x = np.full(32000, np.nan, np.float32)
    s = pkg.Sampler.make(0.0, 0.0, 1.0, 3, pkg.SAMPLER_HOST)
    with pytest.raises(pkg.I4DError):
        ctx.sample(_dev(x).data_ptr(), [], s)  # the host sampler's all-NaN exception
    s = pkg.Sampler.make(0.0, 0.0, 1.0, 3, pkg.SAMPLER_EMULATOR)
    assert ctx.sample(_dev(x).data_ptr(), [], s) == 0  # the emulator's scan stays at index 0
    with pytest.raises(pkg.I4DError):
        ctx.sample(_dev(x).data_ptr(), np.zeros(16385, np.int32), s)  # history limit
    with pytest.raises(pkg.I4DError):
        ctx.sample(_dev(x).data_ptr(), [], pkg.Sampler(temperature=-1.0, top_p=0.0, repeat_penalty=1.0, mode=0))
    # exact ties in the nucleus: candidates in index order
    y = np.full(32000, -30.0, np.float32)
    y[[7, 3, 11, 25000]] = 5.0
    for st in (1, 99, 12345, 2**40 + 3):
        s = pkg.Sampler(temperature=1.0, top_p=0.9, repeat_penalty=1.0, mode=0, rng_state=st)
        assert ctx.sample(_dev(y).data_ptr(), [], s) == oracle.sample(0, y, [], 1.0, 0.9, 1.0, st)[0]


def test_decode_sample_matches_logits_path(pkg, synth, rope_lut, oracle):
    banks, emb = synth.model_banks(LAYERS, SEED), synth.embeddings(SEED)
    with pkg.Context(num_layers=LAYERS, kv_capacity=64) as g, pkg.Context(num_layers=LAYERS, kv_capacity=64) as r:
        for c in (g, r):
            c.load_banks(banks)
            c.load_rope(rope_lut)
        g.load_embeddings(emb)
        s = pkg.Sampler.make(0.8, 0.9, 1.1, 2024, pkg.SAMPLER_HOST)
        st = s.rng_state
        tok, hist = 1, [1]
        for pos in range(8):
            nxt = g.decode_sample(pos, tok, hist, s)
            logits = r.decode_token(pos, emb[tok * 4096:(tok + 1) * 4096])
            want, st = oracle.sample(0, logits[:32000], np.array(hist, np.int32), 0.8, 0.9, 1.1, st)
            assert (nxt, s.rng_state) == (want, st), pos
            tok = nxt
            hist.append(tok)
