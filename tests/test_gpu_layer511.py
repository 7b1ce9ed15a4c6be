"""One decoder layer at position 511 over 511 prior KV records (the
single-layer workload): d_model 4096, 32 heads, FFN 11264, seed 1; the prior
K and V are N(0, 1) values taken to Q15.17 (float_to_q17, emulator:481-505),
K rotated by RoPE at its own position (apply_rope_q17, emulator:526-541) and
both quantised into records by the reference's shift quantiser
(emulator:543-564, 617-631).  The layer input is an N(0, 1) residual.

The same records are written into the GPU context (i4d_kv_write) and into
the reference emulator's cache (oracle/_ref), then one forward() at position
511 runs on both (emulator:727-783: the layer, the final RMSNorm and the LM
head).  Logits, the output residual and the new record at 511 must be
bit-identical."""
import os
import tempfile

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SEED, POS, CAPACITY = 1, 511, 512


def _prior_records(oracle, rope_tables, synth):
    """[bank][lh][token] -> 320-byte record, for tokens 0..POS-1."""
    rng = np.random.default_rng(SEED)
    recs = np.empty((4, 8, POS, 320), np.uint8)
    for t in range(POS):
        k = oracle.float_to_q17(rng.standard_normal(4096).astype(np.float32))
        v = oracle.float_to_q17(rng.standard_normal(4096).astype(np.float32))
        k = oracle.rope(k, rope_tables, t)
        for h in range(32):
            recs[h // 8, h % 8, t] = oracle.kv_record(k[h * 128:(h + 1) * 128], v[h * 128:(h + 1) * 128])
    return recs


def test_layer_at_position_511_matches_reference(pkg, synth, oracle, rope_lut, rope_tables):
    import oracle as orc_mod
    if not orc_mod.ref_available():
        pytest.skip("reference emulator not built (oracle/_ref)")
    banks = synth.model_banks(1, SEED)
    emb = synth.embeddings(SEED)
    x = synth.normal(4096, 0.0, 1.0, SEED, synth.STREAM_INPUT)
    tok = 12345
    emb[tok * 4096:(tok + 1) * 4096] = x  # the emulator's forward() starts from an embedding row
    recs = _prior_records(oracle, rope_tables, synth)

    tmp = "/dev/shm" if os.path.isdir("/dev/shm") else None
    with tempfile.TemporaryDirectory(prefix="i4d_l511_", dir=tmp) as d:
        for p, b in enumerate(banks):
            b.tofile(os.path.join(d, f"model_bank{p}.bin"))
        emb.tofile(os.path.join(d, "embeddings.bin"))
        with open(os.path.join(d, "rope_lut.bin"), "wb") as f:
            f.write(rope_lut)
        ref = orc_mod.RefEmulator()
        ref.load(d, 1, CAPACITY)
    for bank in range(4):
        for lh in range(8):
            for t in range(POS):
                ref.kv_set_record(bank, 0, lh, t, recs[bank, lh, t])
    ref_logits, ref_res = ref.forward(tok, POS)

    with pkg.Context(num_layers=1, kv_capacity=CAPACITY) as ctx:
        ctx.load_banks(banks)
        ctx.load_rope(rope_lut)
        for bank in range(4):
            for lh in range(8):
                for t in range(POS):
                    ctx.kv_write(bank, 0, lh, t, recs[bank, lh, t])
        logits, res = ctx.decode_token(POS, x, want_residual=True)
        new = [[ctx.kv_read(bank, 0, lh, POS) for lh in range(8)] for bank in range(4)]
    assert np.array_equal(logits[:32000].view(np.uint32), ref_logits.view(np.uint32))
    assert np.array_equal(res.view(np.uint32), ref_res.view(np.uint32))
    for bank in range(4):
        for lh in range(8):
            assert np.array_equal(new[bank][lh], ref.kv_record(bank, 0, lh, POS)), (bank, lh)
