"""Batched prefill against the reference emulator itself (oracle/_ref): a
prompt run through i4d_prefill_tokens in batches of up to 32 tokens must leave
the logits the reference's token-by-token prompt loop computes
(decode_host.cpp:1570-1580 drives one forward() per prompt position,
emulator:727-783), bit for bit, and the same KV records of every prompt
position.  Batches of 16 and 32 tokens, a ragged 37-token prompt (32 + 5)
and a prompt continuing after 5 decoded positions; 2 decoder layers."""
import os
import tempfile

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

LAYERS, SEED, CAPACITY = 2, 23, 128


@pytest.fixture(scope="module")
def setup(synth, rope_lut):
    import oracle
    if not oracle.ref_available():
        pytest.skip("reference emulator not built (oracle/_ref)")
    banks = synth.model_banks(LAYERS, SEED)
    emb = synth.embeddings(SEED)
    tmp = "/dev/shm" if os.path.isdir("/dev/shm") else None
    with tempfile.TemporaryDirectory(prefix="i4d_pf_", dir=tmp) as d:
        for p, b in enumerate(banks):
            b.tofile(os.path.join(d, f"model_bank{p}.bin"))
        emb.tofile(os.path.join(d, "embeddings.bin"))
        with open(os.path.join(d, "rope_lut.bin"), "wb") as f:
            f.write(rope_lut)
        ref = oracle.RefEmulator()
        ref.load(d, LAYERS, CAPACITY)
    return banks, emb, ref


@pytest.mark.parametrize("p0,n", [(0, 16), (0, 32), (0, 37), (5, 32)])
def test_prefill_matches_reference_prompt_loop(pkg, rope_lut, setup, p0, n):
    banks, emb, ref = setup
    ids = np.random.default_rng(1000 + 7 * p0 + n).integers(3, 32000, size=p0 + n).astype(np.int32)
    ref.L.ref_kv_reset()
    last = None
    for pos in range(p0 + n):
        last, _ = ref.forward(int(ids[pos]), pos)
    with pkg.Context(num_layers=LAYERS, kv_capacity=CAPACITY) as ctx:
        ctx.load_banks(banks)
        ctx.load_rope(rope_lut)
        ctx.load_embeddings(emb)
        for pos in range(p0):  # an earlier part of the sequence, decoded step by step
            ctx.decode_greedy(pos, int(ids[pos]))
        nxt, logits = ctx.prefill_tokens(p0, ids[p0:], want_logits=True)
        assert np.array_equal(logits[:32000].view(np.uint32), last.view(np.uint32))
        assert nxt == ref.argmax(last)
        for bank in range(4):
            for layer in range(LAYERS):
                for lh in (0, 5):
                    for t in range(p0 + n):
                        assert np.array_equal(ctx.kv_read(bank, layer, lh, t), ref.kv_record(bank, layer, lh, t)), \
                            (bank, layer, lh, t)
