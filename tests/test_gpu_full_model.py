"""Full-size parity (config 3 of the bench: all 32 layers, seed 2): greedy
steps on the GPU against the reference emulator itself (compiled from its
source into oracle/_ref), logits and token ids bit-exact."""
import os
import tempfile

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

PROMPT = [1, 2307, 29871, 13, 31999]
GENERATE = 4


def _write_model(d, banks, emb, lut):
    for p, b in enumerate(banks):
        b.tofile(os.path.join(d, f"model_bank{p}.bin"))
    emb.tofile(os.path.join(d, "embeddings.bin"))
    with open(os.path.join(d, "rope_lut.bin"), "wb") as f:
        f.write(lut)


def test_full_model_greedy_matches_reference_emulator(pkg, synth, rope_lut):
    import oracle
    if not oracle.ref_available():
        pytest.skip("reference emulator not built (oracle/_ref)")
    banks = synth.model_banks(32, 2)
    emb = synth.embeddings(2)
    with pkg.Context(num_layers=32, kv_capacity=64) as ctx:
        ctx.load_banks(banks)
        ctx.load_rope(rope_lut)
        ctx.load_embeddings(emb)
        gpu_ids, gpu_logits = [], []
        tok = PROMPT[0]
        for pos in range(len(PROMPT) + GENERATE):
            nxt, logits = ctx.decode_greedy(pos, tok, want_logits=True)
            gpu_logits.append(logits[:32000].copy())
            gpu_ids.append(nxt)
            tok = PROMPT[pos + 1] if pos + 1 < len(PROMPT) else nxt
    tmp = "/dev/shm" if os.path.isdir("/dev/shm") else None
    with tempfile.TemporaryDirectory(prefix="i4d_full_", dir=tmp) as d:
        _write_model(d, banks, emb, rope_lut)
        ref = oracle.RefEmulator()
        ref.load(d, 32, 64)
        tok = PROMPT[0]
        for pos in range(len(PROMPT) + GENERATE):
            logits, _ = ref.forward(tok, pos)
            assert np.array_equal(logits.view(np.uint32), gpu_logits[pos].view(np.uint32)), pos
            assert ref.argmax(logits) == gpu_ids[pos], pos
            tok = PROMPT[pos + 1] if pos + 1 < len(PROMPT) else gpu_ids[pos]
