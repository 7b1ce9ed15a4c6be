"""On-disk formats of the reference decode path, restated.

* Bank images ``model_bank{0..3}.bin``: 13,516,736 64-byte words each; norm
  words first (kernel_HLS/int4_model_layout.hpp:151-213), then per layer the
  Q, K, V, O, GATE, UP, DOWN superblock streams and finally the LM head
  (autoround_pack_llama2_u250.py:59-99).
* ``rope_lut.bin``: 4096 positions x 64 pairs of signed 19-bit Q1.17
  cosine/sine, 16 pairs per 608-bit word padded to two 64-byte words
  (scripts/generate_rope_lut.py:20-157).
* KV records: 320 bytes per (bank, layer, local head, token): shift word,
  K int8[128], V int8[128] (kernel_HLS/swiftkv_attention.hpp:11-36).
"""
import numpy as np

DIM = 4096
HIDDEN = 11008
FFN = 11264
VOCAB = 32000
PADDED_VOCAB = 32256
HEADS = 32
HEAD_DIM = 128
BANKS = 4
LAYERS = 32
MAX_POSITIONS = 4096
WORD_BYTES = 64
NORM_WORDS = 4160
BANK_WORDS = 13_516_736
BANK_BYTES = BANK_WORDS * WORD_BYTES            # 865,071,104
LEGACY_BANK_BYTES = 891_277_312
SUPERBLOCK_WORDS = 4224
ROPE_BYTES = 2_097_152
KV_RECORD_BYTES = 320

MODE_Q, MODE_K, MODE_V, MODE_O, MODE_GATE, MODE_UP, MODE_DOWN, MODE_LOGITS = range(8)
MODE_NAMES = ["Q", "K", "V", "O", "GATE", "UP", "DOWN", "LOGITS"]

# sha256 of the reference's committed rope_lut.bin (the only binary fixture of
# the reference project); generate_rope_lut() must reproduce it byte for byte.
ROPE_LUT_SHA256 = "29624d3ce00fd843da559f6e141901739ee3e175f11824631d5e934adec49fe9"

# Algorithmic bytes of one token (weights incl. padding, gammas, KV).
W_TOKEN_BYTES = 3_459_219_456                  # data regions of the 4 banks
G_TOKEN_BYTES = 65 * DIM * 4
KV_BYTES_PER_POSITION = 32 * 32 * 261


def mode_rows(mode):
    if mode in (MODE_GATE, MODE_UP):
        return FFN
    if mode == MODE_LOGITS:
        return PADDED_VOCAB
    return DIM


def mode_cols(mode):
    return FFN if mode == MODE_DOWN else DIM


def mode_local_in_tiles(mode):
    return mode_cols(mode) // (BANKS * 256)


def mode_data_words(mode):
    return mode_rows(mode) // 128 * mode_local_in_tiles(mode) // 16 * SUPERBLOCK_WORDS


LAYER_STRIDE_WORDS = sum(mode_data_words(m) for m in range(7))  # 413,952


def matrix_word_offset(layer, mode):
    """Word offset of a matrix inside a bank image (py:88-93, emulator:786-797)."""
    if mode == MODE_LOGITS:
        return NORM_WORDS + LAYERS * LAYER_STRIDE_WORDS
    return NORM_WORDS + layer * LAYER_STRIDE_WORDS + sum(mode_data_words(m) for m in range(mode))


def norm_word_offset(layer, which):
    """0 = attention, 1 = FFN, 2 = final (py:95-99)."""
    if which == 2:
        return LAYERS * 128
    return layer * 128 + (64 if which == 1 else 0)


def token_bytes(position):
    """Algorithmic HBM bytes of one decode step at `position`."""
    return W_TOKEN_BYTES + G_TOKEN_BYTES + KV_BYTES_PER_POSITION * (position + 1)


def generate_rope_lut():
    """rope_lut.bin restated from scripts/generate_rope_lut.py:48-157.

    freq_p = 10000^(-p/64), angle = position * freq_p in float64, values
    rounded half-to-even to Q1.17, saturated to 19 bits, packed LSB-first
    (pair i of a word at bit 38*i: cosine, then sine at +19).
    """
    pos = np.arange(MAX_POSITIONS, dtype=np.float64)
    pairs = np.arange(64, dtype=np.float64)
    freq = 1.0 / (10000.0 ** (pairs / 64))
    ang = np.outer(pos, freq)

    def q17(v):
        raw = np.round(v * (1 << 17)).astype(np.int64)
        raw = np.clip(raw, -(1 << 18), (1 << 18) - 1)
        return (raw & ((1 << 19) - 1)).astype(np.uint64)

    c19 = q17(np.cos(ang)).reshape(MAX_POSITIONS, 4, 16)
    s19 = q17(np.sin(ang)).reshape(MAX_POSITIONS, 4, 16)
    bits = np.zeros((MAX_POSITIONS, 4, 1024), dtype=np.uint8)
    for lane in range(16):
        for f, field in ((0, c19), (1, s19)):
            base = lane * 38 + f * 19
            for b in range(19):
                bits[:, :, base + b] = ((field[:, :, lane] >> np.uint64(b)) & np.uint64(1)).astype(np.uint8)
    return np.packbits(bits, axis=-1, bitorder="little").reshape(-1).tobytes()


def decode_rope_lut(lut):
    """(cos, sin) int32 [4096, 64] from rope_lut.bin bytes (emulator:937-968)."""
    raw = np.frombuffer(lut, dtype=np.uint8).reshape(MAX_POSITIONS, 4, 128)
    bits = np.unpackbits(raw, axis=-1, bitorder="little").astype(np.int64)
    out = []
    for f in range(2):
        vals = np.zeros((MAX_POSITIONS, 4, 16), dtype=np.int64)
        for lane in range(16):
            base = lane * 38 + f * 19
            for b in range(19):
                vals[:, :, lane] |= bits[:, :, base + b] << b
        vals = np.where(vals & (1 << 18), vals - (1 << 19), vals)
        out.append(vals.reshape(MAX_POSITIONS, 64).astype(np.int32))
    return out[0], out[1]


def kv_record_unpack(rec):
    """(k_shift[4], v_shift[4], k int8[128], v int8[128]) of one record."""
    rec = np.frombuffer(bytes(rec), dtype=np.uint8)
    meta = int.from_bytes(rec[:5].tobytes(), "little")
    ks = [(meta >> (5 * g)) & 31 for g in range(4)]
    vs = [(meta >> (20 + 5 * g)) & 31 for g in range(4)]
    return ks, vs, rec[64:192].view(np.int8).copy(), rec[192:320].view(np.int8).copy()
