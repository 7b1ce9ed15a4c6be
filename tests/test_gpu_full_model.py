"""Full-size parity on the decode workload of the benchmark (all 32 layers,
seed 2, KV capacity 2048): a 16-token prompt of ids uniform in [3, 31999],
then 128 greedy ids with no EOS stop, on the GPU against the reference
emulator itself (compiled from its source into oracle/_ref).

The reference loop is generate() (emulator:1608-1682): forward() at
positions 0..15 over the prompt, then one forward per generated id; its
argmax is sample_argmax (emulator:1428-1438).  143 forwards give the 128 ids
(the argmax after positions 15..142).  Every position's 32000 logits must be
bit-identical, and so every id; the KV records of a sample of (bank, layer,
head, position) entries too."""
import os
import tempfile

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SEED = 2
PROMPT_LEN = 16
GENERATE = 128
CAPACITY = 2048


def _write_model(d, banks, emb, lut):
    for p, b in enumerate(banks):
        b.tofile(os.path.join(d, f"model_bank{p}.bin"))
    emb.tofile(os.path.join(d, "embeddings.bin"))
    with open(os.path.join(d, "rope_lut.bin"), "wb") as f:
        f.write(lut)


def test_128_greedy_ids_match_reference_emulator(pkg, synth, rope_lut):
    import oracle
    if not oracle.ref_available():
        pytest.skip("reference emulator not built (oracle/_ref)")
    banks = synth.model_banks(32, SEED)
    emb = synth.embeddings(SEED)
    prompt = np.random.default_rng(SEED).integers(3, 32000, size=PROMPT_LEN).tolist()
    n_pos = PROMPT_LEN + GENERATE - 1
    with pkg.Context(num_layers=32, kv_capacity=CAPACITY) as ctx:
        ctx.load_banks(banks)
        ctx.load_rope(rope_lut)
        ctx.load_embeddings(emb)
        gpu_ids, gpu_logits = [], []
        tok = prompt[0]
        for pos in range(n_pos):
            nxt, logits = ctx.decode_greedy(pos, tok, want_logits=True)
            gpu_logits.append(logits[:32000].copy())
            gpu_ids.append(nxt)
            tok = prompt[pos + 1] if pos + 1 < PROMPT_LEN else nxt
        samples = [(b, l, h, t) for b, l, h, t in [(0, 0, 0, 0), (1, 7, 3, 15), (2, 19, 6, 77), (3, 31, 7, 142),
                                                    (0, 31, 0, 100), (3, 0, 5, 141)]]
        gpu_kv = {k: ctx.kv_read(*k) for k in samples}
    tmp = "/dev/shm" if os.path.isdir("/dev/shm") else None
    with tempfile.TemporaryDirectory(prefix="i4d_full_", dir=tmp) as d:
        _write_model(d, banks, emb, rope_lut)
        del banks  # the emulator holds its own copy of the model
        ref = oracle.RefEmulator()
        ref.load(d, 32, CAPACITY)
    tok = prompt[0]
    ref_ids = []
    for pos in range(n_pos):
        logits, _ = ref.forward(tok, pos)
        assert np.array_equal(logits.view(np.uint32), gpu_logits[pos].view(np.uint32)), pos
        ref_ids.append(ref.argmax(logits))
        assert ref_ids[-1] == gpu_ids[pos], pos
        tok = prompt[pos + 1] if pos + 1 < PROMPT_LEN else ref_ids[-1]
    assert len(ref_ids[PROMPT_LEN - 1:]) == GENERATE
    for k, rec in gpu_kv.items():
        assert np.array_equal(ref.kv_record(*k), rec), k
