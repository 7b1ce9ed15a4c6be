"""Batched prompt prefill against the reference's token-by-token prompt loop
(decode_host.cpp:1570-1580): n prompt tokens through i4d_prefill (up to 16
per pass over the weights) leave the same KV records, bit for bit, as n
decode steps, the last token's logits are bit-equal, and decoding continues
identically after it.  The decode steps are pinned to the oracle by the
other GPU tests (test_gpu_decode.py, test_gpu_token_long.py)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

LAYERS, SEED = 2, 17


@pytest.fixture(scope="module")
def model(synth):
    return synth.model_banks(LAYERS, SEED), synth.embeddings(SEED)


def _pair(pkg, banks, rope_lut, cap, emb=None):
    ctxs = [pkg.Context(num_layers=LAYERS, kv_capacity=cap) for _ in range(2)]
    for c in ctxs:
        c.load_banks(banks)
        c.load_rope(rope_lut)
        if emb is not None:
            c.load_embeddings(emb)
    return ctxs


def _same_kv(a, b, tokens):
    for bank in range(4):
        for layer in range(LAYERS):
            for lh in range(8):
                for t in tokens:
                    ra, rb = a.kv_read(bank, layer, lh, t), b.kv_read(bank, layer, lh, t)
                    assert np.array_equal(ra, rb), (bank, layer, lh, t)


def _u32(x):
    return x.view(np.uint32)


@pytest.mark.parametrize("p0,n", [(0, 37), (5, 16), (3, 1), (0, 70), (2, 24)])
def test_prefill_matches_decode_steps(pkg, rope_lut, model, p0, n):
    banks, _ = model
    rng = np.random.default_rng(SEED + p0 + n)
    x = rng.normal(0.0, 0.02, (p0 + n + 1, 4096)).astype(np.float32)
    pf, dec = _pair(pkg, banks, rope_lut, 128)
    with pf, dec:
        for pos in range(p0):  # an earlier part of the sequence, decoded on both
            assert np.array_equal(_u32(pf.decode_token(pos, x[pos])), _u32(dec.decode_token(pos, x[pos])))
        last = None
        for pos in range(p0, p0 + n):
            last = dec.decode_token(pos, x[pos])
        lp = pf.prefill(p0, x[p0:p0 + n])
        assert np.array_equal(_u32(lp), _u32(last))
        _same_kv(pf, dec, range(p0 + n))
        nxt = p0 + n
        assert np.array_equal(_u32(pf.decode_token(nxt, x[nxt])), _u32(dec.decode_token(nxt, x[nxt])))


def test_prefill_tokens_matches_greedy(pkg, rope_lut, model):
    banks, emb = model
    ids = np.random.default_rng(3).integers(0, 32000, 21).astype(np.int32)
    pf, dec = _pair(pkg, banks, rope_lut, 64, emb)
    with pf, dec:
        for pos, tok in enumerate(ids):
            nxt_d, logits_d = dec.decode_greedy(pos, int(tok), want_logits=True)
        nxt_p, logits_p = pf.prefill_tokens(0, ids, want_logits=True)
        assert nxt_p == nxt_d
        assert np.array_equal(_u32(logits_p), _u32(logits_d))
        _same_kv(pf, dec, range(len(ids)))
        a, _ = pf.decode_greedy(len(ids), nxt_p)
        b, _ = dec.decode_greedy(len(ids), nxt_d)
        assert a == b


def test_prefill_rejects_bad_arguments(pkg, rope_lut, model):
    banks, emb = model
    with pkg.Context(num_layers=LAYERS, kv_capacity=32) as c:
        c.load_banks(banks)
        c.load_rope(rope_lut)
        x = np.zeros((4, 4096), np.float32)
        with pytest.raises(pkg.I4DError):
            c.prefill(30, x)  # positions 30..33 beyond the capacity
        with pytest.raises(pkg.I4DError):
            c.prefill_tokens(0, [1, 2])  # no embeddings loaded
        c.load_embeddings(emb)
        with pytest.raises(pkg.I4DError):
            c.prefill_tokens(0, [1, 32000])
        with pytest.raises(pkg.I4DError):
            c.prefill_tokens(0, np.zeros(0, np.int32))
        # the context still decodes after the refusals
        c.prefill(0, x)
