"""Token-level parity of i4d_decode_token against the CPU oracle (bit-exact)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

LAYERS = 2
SEED = 11


@pytest.fixture(scope="module")
def model(synth):
    banks = synth.model_banks(LAYERS, SEED)
    emb = synth.embeddings(SEED)
    return banks, emb


def _oracle_steps(oracle, rope_tables, banks, emb, tokens, stride):
    kv = oracle.kv_store(LAYERS, stride)
    outs = []
    for pos, tok in enumerate(tokens):
        logits, res = oracle.forward(banks, rope_tables, kv, LAYERS, stride, pos, emb[tok * 4096:(tok + 1) * 4096])
        outs.append((logits, res))
    return outs, kv


@pytest.fixture(scope="module")
def reference_run(oracle, rope_tables, model):
    banks, emb = model
    tokens = [1, 29871, 13, 450, 31999, 7, 3, 100]
    outs, kv = _oracle_steps(oracle, rope_tables, banks, emb, tokens, 64)
    return tokens, outs, kv


# 0: persistent token kernel in a graph; 1: persistent, eager; 4: one kernel
# per stage (graph + PDL); 5: staged, eager; 6: staged without PDL
@pytest.mark.parametrize("flags", [0, 1, 4, 5, 6])
def test_decode_bit_exact(pkg, model, rope_lut, reference_run, flags):
    banks, emb = model
    tokens, outs, kv = reference_run
    with pkg.Context(num_layers=LAYERS, kv_capacity=64, flags=flags) as ctx:
        ctx.load_banks(banks)
        ctx.load_rope(rope_lut)
        for pos, tok in enumerate(tokens):
            logits, res = ctx.decode_token(pos, emb[tok * 4096:(tok + 1) * 4096], want_residual=True)
            ologits, ores = outs[pos]
            assert np.array_equal(res.view(np.uint32), ores.view(np.uint32)), pos
            assert np.array_equal(logits, ologits), pos
            assert int(np.argmax(logits[:32000])) == int(np.argmax(ologits[:32000]))
        for bank, layer, lh, tok in [(0, 0, 0, 0), (3, 1, 7, 7), (1, 1, 2, 4)]:
            rec = ctx.kv_read(bank, layer, lh, tok)
            off = ((((bank * LAYERS) + layer) * 8 + lh) * 64 + tok) * 320
            assert np.array_equal(rec, kv[off:off + 320])


def test_decode_rejects_bad_calls(pkg, model, rope_lut, F):
    banks, emb = model
    with pkg.Context(num_layers=1, kv_capacity=8) as ctx:
        with pytest.raises(pkg.I4DError) as e:
            ctx.decode_token(0, emb[:4096])
        assert e.value.status == pkg.ERR_STATE
        with pytest.raises(pkg.I4DError) as e:
            ctx._check(ctx._L.i4d_load_bank(ctx._h, 0, banks[0].ctypes.data, F.LEGACY_BANK_BYTES))
        assert e.value.status == pkg.ERR_SIZE
        with pytest.raises(pkg.I4DError) as e:
            ctx._check(ctx._L.i4d_load_bank(ctx._h, 0, banks[0].ctypes.data, F.BANK_BYTES - 64))
        assert e.value.status == pkg.ERR_SIZE
        ctx.load_banks(banks)
        ctx.load_rope(rope_lut)
        with pytest.raises(pkg.I4DError) as e:
            ctx.decode_token(8, emb[:4096])
        assert e.value.status == pkg.ERR_ARG
        ctx.decode_token(0, emb[:4096])  # the context stays usable
