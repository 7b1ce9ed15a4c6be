"""The perplexity term of the oracle (i4o_nll, emulator:1902-1926) pinned to
the reference's own calculate_perplexity (emulator:1775-1958), compiled from
its source into oracle/_ref: on a 1-layer synthetic model and a seeded token
file, the oracle's terms over the reference emulator's own logits give the
token count, loss and PPL that the reference prints."""
import math
import os
import re
import tempfile

import numpy as np
import pytest

LAYERS, SEED, N = 1, 23, 12


def _write_model(d, banks, emb, lut):
    for p, b in enumerate(banks):
        b.tofile(os.path.join(d, f"model_bank{p}.bin"))
    emb.tofile(os.path.join(d, "embeddings.bin"))
    with open(os.path.join(d, "rope_lut.bin"), "wb") as f:
        f.write(lut)


def test_oracle_nll_reproduces_reference_perplexity(synth, rope_lut, oracle, capfd):
    import oracle as orc
    if not orc.ref_available():
        pytest.skip("reference emulator not built (oracle/_ref)")
    banks = synth.model_banks(LAYERS, SEED)
    emb = synth.embeddings(SEED)
    ids = np.random.default_rng(SEED).integers(3, 32000, N).astype(np.int32)
    tmp = "/dev/shm" if os.path.isdir("/dev/shm") else None
    with tempfile.TemporaryDirectory(prefix="i4d_ppl_", dir=tmp) as d:
        _write_model(d, banks, emb, rope_lut)
        ref = orc.RefEmulator()
        ref.load(d, LAYERS, 64)
        path = os.path.join(d, "tokens.bin")
        ids.tofile(path)
        capfd.readouterr()
        ref.perplexity(path)
        out = capfd.readouterr().out
        total = 0.0
        for pos in range(N - 1):
            logits, _ = ref.forward(int(ids[pos]), pos)
            total += oracle.nll(logits, int(ids[pos + 1]))[0]
    loss = total / (N - 1)
    assert re.search(r"Total Tokens Evaluated\s*:\s*(\d+)", out).group(1) == str(N - 1)
    assert re.search(r"Average Cross-Entropy\s*:\s*([0-9.]+)", out).group(1) == f"{loss:.4f}"
    assert re.search(r"Perplexity \(PPL\)\s*:\s*([0-9.]+)", out).group(1) == f"{math.exp(loss):.2f}"


def test_oracle_nll_edge_cases(oracle):
    x = np.full(32000, -3.0, np.float32)
    x[5] = 2.0
    v, m, s = oracle.nll(x, 5)
    assert m == 2.0 and s > 1.0 and v > 0.0
    y = x.copy()
    y[0] = np.nan  # the serial maximum starts at a NaN and stays NaN
    v, m, s = oracle.nll(y, 5)
    assert math.isnan(m) and math.isnan(v)
    z = x.copy()
    z[7] = np.nan  # a later NaN is never taken as the maximum but poisons the sum
    v, m, s = oracle.nll(z, 5)
    assert m == 2.0 and math.isnan(s)
