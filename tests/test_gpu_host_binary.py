"""The C++ host (i4d_decode, the decode_host drop-in) on a model directory in
the reference's file formats: the prompt through i4d_prefill (--prefill)
gives the same greedy continuation as the reference's one-token-per-step
prompt loop (decode_host.cpp:1570-1580)."""
import os
import subprocess
import tempfile

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BIN = os.path.join(ROOT, "4pe_u250_b200", "i4d_decode")
LAYERS, SEED = 2, 31


def _write_model(d, banks, emb, lut):
    for p, b in enumerate(banks):
        b.tofile(os.path.join(d, f"model_bank{p}.bin"))
    emb.tofile(os.path.join(d, "embeddings.bin"))
    with open(os.path.join(d, "rope_lut.bin"), "wb") as f:
        f.write(lut)


def _generated(out):
    line = [ln for ln in out.splitlines() if ln.startswith("[Generated token IDs]")][0]
    return [int(x) for x in line.split("]")[1].split()]


def test_host_binary_prefill_matches_per_token_prompt(synth, rope_lut):
    if not os.path.exists(BIN):
        pytest.fail(f"{BIN} missing: run __graft_entry__.build()")
    banks = synth.model_banks(LAYERS, SEED)
    emb = synth.embeddings(SEED)
    prompt = ",".join(str(int(t)) for t in np.random.default_rng(SEED).integers(3, 32000, 21))
    tmp = "/dev/shm" if os.path.isdir("/dev/shm") else None
    with tempfile.TemporaryDirectory(prefix="i4d_host_", dir=tmp) as d:
        _write_model(d, banks, emb, rope_lut)
        args = [BIN, "--banks", d, "--prompt-ids", prompt, "--layers", str(LAYERS), "--kv-capacity", "64",
                "--max-tokens", "6", "--no-eos"]
        ref = subprocess.run(args, capture_output=True, text=True, timeout=300)
        pf = subprocess.run(args + ["--prefill"], capture_output=True, text=True, timeout=300)
    assert ref.returncode == 0, ref.stderr
    assert pf.returncode == 0, pf.stderr
    assert len(_generated(ref.stdout)) == 6
    assert _generated(pf.stdout) == _generated(ref.stdout)
