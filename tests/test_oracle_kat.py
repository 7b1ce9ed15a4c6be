"""Pins the CPU oracle against the reference's own known-answer tests."""
import numpy as np
import pytest

import kat_vectors as K


@pytest.mark.parametrize("mode,out_tiles,pattern", K.LINEAR_CASES)
def test_linear_kat_bit_exact(oracle, mode, out_tiles, pattern):
    model, lit, q, e, expected = K.linear_case(mode, out_tiles, pattern)
    got = oracle.linear_bank(model, out_tiles, lit, q, e, hls_zero_start=True)
    assert got.view(np.uint32).tolist() == expected.view(np.uint32).tolist()


def test_linear_kat_emulator_zero_convention(oracle):
    """The emulator starts each chain at +0.0f: only the sign of all-zero sums differs."""
    model, lit, q, e, expected = K.linear_case("O", 4, 2)
    got = oracle.linear_bank(model, 4, lit, q, e, hls_zero_start=False)
    assert np.array_equal(got, expected)  # -0.0 == +0.0
    assert (np.signbit(expected)).any() and not np.signbit(got).any()


def _pe0_attention(oracle, rope_tables, kv, pos, seeds):
    full = []
    for s in seeds:
        v = np.zeros(4096, np.int32)
        v[:1024] = K.pe0_vector(s)
        full.append(v)
    q = oracle.rope(full[0], rope_tables, pos)
    k = oracle.rope(full[1], rope_tables, pos)
    return oracle.attention(kv, 1, 3, 0, pos, q, k, full[2])


def test_attention_pe0_fnv_hashes(oracle, rope_tables):
    kv = oracle.kv_store(1, 3)
    q0, e0 = _pe0_attention(oracle, rope_tables, kv, 0, K.ATTN_SEEDS[0])
    q1, e1 = _pe0_attention(oracle, rope_tables, kv, 1, K.ATTN_SEEDS[1])
    assert K.fnv_hash_pe0(q0, e0) == K.ATTN_HASH_POS0
    assert K.fnv_hash_pe0(q1, e1) == K.ATTN_HASH_POS1
