"""Format constants and the RoPE LUT fixture."""
import hashlib
import os

import numpy as np


def test_rope_lut_matches_reference_fixture(F, rope_lut):
    assert len(rope_lut) == F.ROPE_BYTES
    assert hashlib.sha256(rope_lut).hexdigest() == F.ROPE_LUT_SHA256
    # With the reference tree at hand (I4D_REF_ROOT), also its committed file.
    root = os.environ.get("I4D_REF_ROOT")
    ref = os.path.join(root, "rope_lut.bin") if root else None
    if ref and os.path.exists(ref):
        assert open(ref, "rb").read() == rope_lut


def test_rope_decode_round_trip(F, rope_lut, rope_tables):
    c, s = F.decode_rope_lut(rope_lut)
    oc, os_ = rope_tables
    assert np.array_equal(c.reshape(-1), oc) and np.array_equal(s.reshape(-1), os_)
    # position 0: cos = 1.0 (131072), sin = 0
    assert (c[0] == 131072).all() and (s[0] == 0).all()


def test_bank_layout_constants(F):
    assert F.BANK_BYTES == 865_071_104
    assert F.LAYER_STRIDE_WORDS == 413_952
    assert [F.mode_data_words(m) for m in range(8)] == [33792] * 4 + [92928] * 3 + [266112]
    assert F.matrix_word_offset(0, F.MODE_LOGITS) == 4160 + 13_246_464
    assert F.matrix_word_offset(0, F.MODE_LOGITS) + 266112 == F.BANK_WORDS
    assert F.matrix_word_offset(1, F.MODE_K) == 4160 + 413_952 + 33_792
    assert F.norm_word_offset(3, 1) == 3 * 128 + 64 and F.norm_word_offset(0, 2) == 4096
    assert F.W_TOKEN_BYTES + F.G_TOKEN_BYTES == 4 * F.BANK_BYTES


def test_token_bytes(F):
    assert F.token_bytes(0) == 3_459_219_456 + 1_064_960 + 267_264
