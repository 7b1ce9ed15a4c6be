"""Perplexity on the device: per-position negative
log-likelihoods from prompt batches (i4d_eval_nll) bit-equal, as doubles, to
the oracle's term (i4o_nll, pinned to the reference's calculate_perplexity in
test_ppl_oracle.py) over the decode path's logits, and the chunked loop of
Context.perplexity equal to the same loop over those terms."""
import math

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

LAYERS, SEED = 2, 29


@pytest.fixture(scope="module")
def model(synth):
    return synth.model_banks(LAYERS, SEED), synth.embeddings(SEED)


def _ctx(pkg, banks, rope_lut, emb, cap=64):
    c = pkg.Context(num_layers=LAYERS, kv_capacity=cap)
    c.load_banks(banks)
    c.load_rope(rope_lut)
    c.load_embeddings(emb)
    return c


def _oracle_chunk(dec, oracle, emb, ids):
    out = []
    for pos in range(len(ids) - 1):
        t = int(ids[pos])
        logits = dec.decode_token(pos, emb[t * 4096:(t + 1) * 4096])
        out.append(oracle.nll(logits[:32000], int(ids[pos + 1]))[0])
    return np.array(out, np.float64)


def test_eval_nll_matches_oracle(pkg, rope_lut, oracle, model):
    banks, emb = model
    ids = np.random.default_rng(SEED).integers(3, 32000, 40).astype(np.int32)
    with _ctx(pkg, banks, rope_lut, emb) as g, _ctx(pkg, banks, rope_lut, emb) as dec:
        got = g.eval_nll(ids)
        want = _oracle_chunk(dec, oracle, emb, ids)
        assert got.shape == (39,)
        assert np.array_equal(got.view(np.uint64), want.view(np.uint64))
        two = g.eval_nll(ids[:2])
        assert np.array_equal(two.view(np.uint64), want[:1].view(np.uint64))


def test_perplexity_loop_matches_oracle(pkg, rope_lut, oracle, model):
    banks, emb = model
    ids = np.random.default_rng(SEED + 1).integers(3, 32000, 45).astype(np.int32)
    with _ctx(pkg, banks, rope_lut, emb) as g, _ctx(pkg, banks, rope_lut, emb) as dec:
        loss, ppl, count = g.perplexity(ids, chunk=20)
        total, n = 0.0, 0
        for start in range(0, ids.size, 20):
            part = ids[start:start + 20]
            if part.size < 2:
                break
            for v in _oracle_chunk(dec, oracle, emb, part):
                total += float(v)
                n += 1
        assert count == n == 19 + 19 + 4
        assert loss == total / n and ppl == math.exp(total / n)


def test_eval_nll_rejects_bad_input(pkg, rope_lut, model):
    banks, emb = model
    with _ctx(pkg, banks, rope_lut, emb, cap=16) as g:
        with pytest.raises(pkg.I4DError):
            g.eval_nll([5])
        with pytest.raises(pkg.I4DError):
            g.eval_nll([5, 32000])
        with pytest.raises(pkg.I4DError):
            g.eval_nll(np.arange(3, 21, dtype=np.int32))  # 17 positions beyond a capacity of 16
        assert g.eval_nll(np.arange(3, 20, dtype=np.int32)).shape == (16,)
