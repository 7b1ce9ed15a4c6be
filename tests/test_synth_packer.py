"""The synthetic generator writes the reference's bank format exactly."""
import hashlib
import importlib.util
import json
import os

import numpy as np
import pytest

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "packer_golden.json")
REF_ROOT = os.environ.get("I4D_REF_ROOT")
REF_PACKER = os.path.join(REF_ROOT, "scripts", "autoround_pack_llama2_u250.py") if REF_ROOT else ""


def _small_case():
    rng = np.random.default_rng(123)
    M, K = 512, 4096
    w = rng.integers(-8, 8, size=(M, K), dtype=np.int8)
    s = rng.integers(66, 656, size=(M, K // 128)).astype(np.int16)
    return w, s, M, K


@pytest.mark.skipif(not os.path.exists(REF_PACKER), reason="I4D_REF_ROOT does not name a reference tree")
def test_c_packer_matches_reference_python_packer(synth):
    spec = importlib.util.spec_from_file_location("ref_packer", REF_PACKER)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    w, s, M, K = _small_case()
    for bank in range(4):
        ref = mod.pack_matrix_to_super_blocks(bank, w, s, M // 128, K // 1024, M, K)
        mine = synth.pack_arrays(w, s, bank, M // 128, K // 1024)
        assert np.array_equal(ref, mine), bank


def test_c_packer_golden_digest(synth):
    w, s, M, K = _small_case()
    golden = json.load(open(GOLDEN))
    for bank in range(4):
        mine = synth.pack_arrays(w, s, bank, M // 128, K // 1024)
        assert hashlib.sha256(mine.tobytes()).hexdigest() == golden["pack_arrays"][str(bank)]


def test_synthetic_matrix_round_trip(synth, oracle, F):
    """fill_matrix packs i4s_weight/i4s_scale values; the oracle GEMV over them
    equals a dense float64 reference within FP32 rounding."""
    banks = synth.empty_banks()
    synth.fill_matrix(banks, 0, F.MODE_O, 5)
    W = synth.weight_matrix(5, 0, F.MODE_O, rows=64)
    x = synth.normal(4096, 0.0, 1.0, 5, synth.STREAM_INPUT)
    q, e = oracle.quantize_g32(x)
    y, _ = oracle.gemv(banks, 0, F.MODE_O, q, e)
    L = synth.lib()
    sc = np.array([[L.i4s_scale(5, 0, F.MODE_O, r, g) for g in range(32)] for r in range(64)]) / 32768.0
    xs = q.astype(np.float64) * np.ldexp(1.0, e.astype(np.int64) - 140).repeat(32)
    ref = (W.astype(np.float64) * np.repeat(sc, 128, axis=1) * xs).sum(axis=1)
    assert np.allclose(y[:64], ref, rtol=1e-4, atol=1e-4 * np.abs(ref).max())
