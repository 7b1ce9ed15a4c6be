"""Per-stage parity of the CUDA path against the CPU oracle (bit-exact)."""
import os
import re

import numpy as np
import pytest

import kat_vectors as K

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _bits(a):
    return np.ascontiguousarray(a).view(np.uint32)


@pytest.fixture(scope="module")
def banks(synth):
    return synth.model_banks(2, 7)


@pytest.fixture(scope="module")
def ctx(pkg, banks, rope_lut):
    c = pkg.Context(num_layers=2, kv_capacity=4096)
    c.load_banks(banks)
    c.load_rope(rope_lut)
    yield c
    c.close()


def _exception_keys():
    path = os.path.join(ROOT, "4pe_u250_b200", "csrc", "gen", "expf_fix_table.c")
    text = open(path).read()
    vals = [int(v, 16) for v in re.findall(r"0x([0-9a-f]{8})u", text)]
    return np.array(vals[0::2], dtype=np.uint32)


def test_expf_matches_host_libc(ctx, oracle):
    rng = np.random.default_rng(0)
    keys = _exception_keys()
    rnd = rng.uniform(-110.0, 100.0, size=4_000_000).astype(np.float32)
    small = (rng.standard_normal(2_000_000) * rng.choice([1e-8, 1e-3, 1.0, 20.0], 2_000_000)).astype(np.float32)
    bits = rng.integers(0, 2**32, size=2_000_000, dtype=np.uint64).astype(np.uint32).view(np.float32)
    special = np.array([0.0, -0.0, np.inf, -np.inf, 88.72283, 88.72284, -103.97208, -87.33655, 1e-45, -1e-45,
                        2**-24, -2**-24, 2**-25], dtype=np.float32)
    x = np.concatenate([keys.view(np.float32), rnd, small, bits, special])
    x = x[~np.isnan(x)]
    got = ctx.expf(x)
    want = oracle.expf(x)
    bad = np.nonzero(_bits(got) != _bits(want))[0]
    assert bad.size == 0, f"{bad.size} mismatches, e.g. x={x[bad[:5]]} got={got[bad[:5]]} want={want[bad[:5]]}"


def test_quantize_g32(ctx, oracle):
    rng = np.random.default_rng(1)
    parts = [rng.standard_normal(4096), rng.standard_normal(4096) * 1e-40, np.zeros(64),
             rng.standard_normal(4096) * 1e30, -np.abs(rng.standard_normal(4096)),
             np.where(rng.random(4096) < 0.5, 0.0, rng.standard_normal(4096) * 1e-20)]
    x = np.concatenate(parts).astype(np.float32)
    x = x[: x.size // 32 * 32]
    gq, ge = ctx.quantize_g32(x)
    oq, oe = oracle.quantize_g32(x)
    assert np.array_equal(gq, oq) and np.array_equal(ge, oe)


@pytest.mark.parametrize("scale", [1.0, 1e-3, 40.0])
def test_rms_quant(ctx, oracle, synth, scale):
    x = synth.normal(4096, 0.0, scale, 3, 11)
    g = synth.normal(4096, 1.0, 0.05, 3, 12)
    gq, ge = ctx.rms_quant(x, g)
    oq, oe, _ = oracle.rms_quant(x, g)
    assert np.array_equal(gq, oq) and np.array_equal(ge, oe)


def test_swiglu_quant(ctx, oracle, synth):
    gate = synth.normal(11264, 0.0, 4.0, 4, 1)
    up = synth.normal(11264, 0.0, 2.0, 4, 2)
    keys = _exception_keys().view(np.float32)
    gate[:4096] = -keys[np.random.default_rng(2).choice(keys.size, 4096)]  # exercise the table
    gq, ge = ctx.swiglu_quant(gate, up)
    oq, oe = oracle.quantize_g32(oracle.swiglu(gate, up))
    assert np.array_equal(gq, oq) and np.array_equal(ge, oe)


@pytest.mark.parametrize("mode,out_tiles,pattern", K.LINEAR_CASES)
def test_linear_bank_kat(ctx, oracle, mode, out_tiles, pattern):
    model, lit, q, e, expected = K.linear_case(mode, out_tiles, pattern)
    got = ctx.linear_bank(model, lit, out_tiles, q, e, hls_zero_start=True)
    assert _bits(got).tolist() == _bits(expected).tolist()
    emu = ctx.linear_bank(model, lit, out_tiles, q, e, hls_zero_start=False)
    assert _bits(emu).tolist() == _bits(oracle.linear_bank(model, out_tiles, lit, q, e)).tolist()


@pytest.mark.parametrize("layer,mode", [(0, m) for m in range(8)] + [(1, 0), (1, 6)])
def test_gemv_bit_exact(ctx, oracle, banks, synth, F, layer, mode):
    x = synth.normal(F.mode_cols(mode), 0.0, 1.0, 100 + mode, synth.STREAM_INPUT)
    q, e = oracle.quantize_g32(x)
    y, part = ctx.gemv(layer, mode, q, e, with_partials=True)
    oy, opart = oracle.gemv(banks, layer, mode, q, e)
    assert _bits(part).tolist() == _bits(opart).tolist()
    assert _bits(y).tolist() == _bits(oy).tolist()


def test_attention_pe0_fnv_hashes(pkg, rope_lut):
    c = pkg.Context(num_layers=1, kv_capacity=3)
    c.load_rope(rope_lut)
    hashes = []
    for pos in (0, 1):
        vecs = []
        for s in K.ATTN_SEEDS[pos]:
            v = np.zeros(4096, np.int32)
            v[:1024] = K.pe0_vector(s)
            vecs.append(v)
        q, e = c.attention(0, pos, *vecs)
        hashes.append(K.fnv_hash_pe0(q, e))
    c.close()
    assert hashes == [K.ATTN_HASH_POS0, K.ATTN_HASH_POS1]


def _rand_q17(rng, n, scale):
    return np.round(rng.standard_normal(n) * scale * 131072).astype(np.int32)


def test_attention_sequence(ctx, oracle, rope_tables):
    """Positions 0..47 of layer 1 with fresh Q/K/V each step; output and KV records."""
    rng = np.random.default_rng(5)
    ctx.kv_reset()
    kv = oracle.kv_store(2, 4096)
    for pos in range(48):
        q, k, v = (_rand_q17(rng, 4096, s) for s in (1.0, 1.0, 0.5))
        gq, ge = ctx.attention(1, pos, q, k, v)
        oq, oe = oracle.attention(kv, 2, 4096, 1, pos, oracle.rope(q, rope_tables, pos),
                                  oracle.rope(k, rope_tables, pos), v)
        assert np.array_equal(gq, oq) and np.array_equal(ge, oe), pos
    for bank, lh, tok in [(0, 0, 0), (1, 3, 17), (3, 7, 47), (2, 5, 30)]:
        rec = ctx.kv_read(bank, 1, lh, tok)
        off = ((((bank * 2) + 1) * 8 + lh) * 4096 + tok) * 320
        assert np.array_equal(rec, kv[off:off + 320]), (bank, lh, tok)


@pytest.mark.parametrize("length", [512, 1024, 2048, 4096])
def test_attention_long_context(ctx, oracle, rope_tables, length):
    """Attention sweep (config 4): `length-1` prior K/V records, decode at length-1."""
    rng = np.random.default_rng(length)
    kv = oracle.kv_store(2, 4096)
    pos = length - 1
    for bank in range(4):
        for lh in range(8):
            ks = _rand_q17(rng, 128 * pos, 1.0).reshape(pos, 128)
            vs = _rand_q17(rng, 128 * pos, 1.0).reshape(pos, 128)
            base = (((bank * 2) + 0) * 8 + lh) * 4096 * 320
            for t in range(pos):
                kv[base + t * 320: base + (t + 1) * 320] = oracle.kv_record(ks[t], vs[t])
    # one device write of the whole layer-0 region through the record API
    for bank in range(4):
        for lh in range(8):
            base = (((bank * 2) + 0) * 8 + lh) * 4096 * 320
            for t in range(pos):
                ctx.kv_write(bank, 0, lh, t, kv[base + t * 320: base + (t + 1) * 320])
    q, k, v = (_rand_q17(rng, 4096, s) for s in (1.0, 1.0, 1.0))
    gq, ge = ctx.attention(0, pos, q, k, v)
    oq, oe = oracle.attention(kv, 2, 4096, 0, pos, oracle.rope(q, rope_tables, pos),
                              oracle.rope(k, rope_tables, pos), v)
    assert np.array_equal(gq, oq) and np.array_equal(ge, oe)


def _write_records(ctx, kv, layer, records_by_head):
    for head, recs in records_by_head.items():
        bank, lh = divmod(head, 8)
        base = (((bank * 2) + layer) * 8 + lh) * 4096 * 320
        for t, rec in enumerate(recs):
            kv[base + t * 320: base + (t + 1) * 320] = rec
            ctx.kv_write(bank, layer, lh, t, rec)


def _record(k8, ks, v8, vs):
    rec = np.zeros(320, np.uint8)
    meta = 0
    for g in range(4):
        meta |= (ks[g] & 31) << (5 * g)
        meta |= (vs[g] & 31) << (20 + 5 * g)
    rec[:5] = np.frombuffer(meta.to_bytes(8, "little")[:5], np.uint8)
    rec[64:192] = np.asarray(k8, np.int8).view(np.uint8)
    rec[192:320] = np.asarray(v8, np.int8).view(np.uint8)
    return rec


def test_attention_many_rescale_events(ctx, oracle, rope_tables):
    """Scores that rise every other token: more than 16 rescale events, so the
    kernel takes its fully sequential path."""
    rng = np.random.default_rng(9)
    ctx.kv_reset()
    pos = 40
    q = rng.integers(-1024, 1024, 4096).astype(np.int32)
    qr = oracle.rope(q, rope_tables, pos)
    kv = oracle.kv_store(2, 4096)
    recs = {}
    for head in (0, 9, 31):
        k8 = np.where(qr[head * 128:(head + 1) * 128] >= 0, 100, -100)
        recs[head] = [_record(k8, [10 + t // 2] * 4, rng.integers(-127, 128, 128), [3] * 4) for t in range(pos)]
    _write_records(ctx, kv, 1, recs)
    k, v = (_rand_q17(rng, 4096, 0.01) for _ in range(2))
    gq, ge = ctx.attention(1, pos, q, k, v)
    oq, oe = oracle.attention(kv, 2, 4096, 1, pos, qr, oracle.rope(k, rope_tables, pos), v)
    assert np.array_equal(gq, oq) and np.array_equal(ge, oe)


def test_attention_saturating_state(ctx, oracle, rope_tables):
    """Equal scores and large values: the per-step int32 saturation of the
    state chain triggers, so the kernel replays the segment sequentially."""
    rng = np.random.default_rng(10)
    ctx.kv_reset()
    pos = 60
    kv = oracle.kv_store(2, 4096)
    recs = {}
    for head in (1, 17):
        k8 = rng.integers(-5, 6, 128)
        recs[head] = [_record(k8, [2] * 4, [100] * 128, [24] * 4) for _ in range(pos)]
    _write_records(ctx, kv, 0, recs)
    q, k, v = (_rand_q17(rng, 4096, 0.01) for _ in range(3))
    gq, ge = ctx.attention(0, pos, q, k, v)
    oq, oe = oracle.attention(kv, 2, 4096, 0, pos, oracle.rope(q, rope_tables, pos),
                              oracle.rope(k, rope_tables, pos), v)
    assert np.array_equal(gq, oq) and np.array_equal(ge, oe)


@pytest.mark.parametrize("pos", [100, 127, 128, 200, 255, 256, 257, 520])
def test_attention_rising_scores(ctx, oracle, rope_tables, pos):
    """Scores that rise on most tokens (a new maximum nearly every step, as a
    recency-biased head gives): more events than a 256-token window applies as
    a chain, so those windows go token by token; positions on both sides of
    a window boundary (the current token first or last in its window)."""
    rng = np.random.default_rng(11 + pos)
    ctx.kv_reset()
    q = rng.integers(-1024, 1024, 4096).astype(np.int32)
    qr = oracle.rope(q, rope_tables, pos)
    kv = oracle.kv_store(2, 4096)
    recs = {}
    for head in (2, 13, 30):
        k8 = np.where(qr[head * 128:(head + 1) * 128] >= 0, 60, -60)
        recs[head] = [_record(k8, [4 + (t * 20) // pos + (t % 3 == 0)] * 4, rng.integers(-127, 128, 128),
                              [int(rng.integers(0, 14))] * 4) for t in range(pos)]
    _write_records(ctx, kv, 1, recs)
    k, v = (_rand_q17(rng, 4096, 0.5) for _ in range(2))
    gq, ge = ctx.attention(1, pos, q, k, v)
    oq, oe = oracle.attention(kv, 2, 4096, 1, pos, qr, oracle.rope(k, rope_tables, pos), v)
    assert np.array_equal(gq, oq) and np.array_equal(ge, oe)


def test_attention_saturation_in_a_later_tile(ctx, oracle, rope_tables):
    """Small values in the first tile, then values near the int32 limit from
    token 150 on: the windows after the first take the saturating path."""
    rng = np.random.default_rng(12)
    ctx.kv_reset()
    pos = 230
    kv = oracle.kv_store(2, 4096)
    recs = {}
    for head in (4, 21):
        k8 = rng.integers(-5, 6, 128)
        recs[head] = [_record(k8, [2] * 4, rng.integers(-127, 128, 128), [24 if t >= 150 else 6] * 4)
                      for t in range(pos)]
    _write_records(ctx, kv, 0, recs)
    q, k, v = (_rand_q17(rng, 4096, 0.01) for _ in range(3))
    gq, ge = ctx.attention(0, pos, q, k, v)
    oq, oe = oracle.attention(kv, 2, 4096, 0, pos, oracle.rope(q, rope_tables, pos),
                              oracle.rope(k, rope_tables, pos), v)
    assert np.array_equal(gq, oq) and np.array_equal(ge, oe)


@pytest.mark.parametrize("pos", [150, 300, 700])
def test_attention_events_across_warps(ctx, oracle, rope_tables, pos):
    """A moderate number of events per window (the shift steps up every few
    tokens, with one-token bumps between): the windows take the summed path
    with runs that start in one worker warp's 16 tokens and end in a later
    one, and events inside a warp's tokens."""
    rng = np.random.default_rng(20 + pos)
    ctx.kv_reset()
    q = rng.integers(-1024, 1024, 4096).astype(np.int32)
    qr = oracle.rope(q, rope_tables, pos)
    kv = oracle.kv_store(2, 4096)
    recs = {}
    for head in (3, 18, 29):
        k8 = np.where(qr[head * 128:(head + 1) * 128] >= 0, 40, -40)
        recs[head] = [_record(k8, [2 + (t * 12) // pos + (t % 11 == 5)] * 4, rng.integers(-127, 128, 128),
                              [int(rng.integers(0, 10))] * 4) for t in range(pos)]
    _write_records(ctx, kv, 1, recs)
    k, v = (_rand_q17(rng, 4096, 0.5) for _ in range(2))
    gq, ge = ctx.attention(1, pos, q, k, v)
    oq, oe = oracle.attention(kv, 2, 4096, 1, pos, qr, oracle.rope(k, rope_tables, pos), v)
    assert np.array_equal(gq, oq) and np.array_equal(ge, oe)


def test_attention_saturation_in_a_later_window(ctx, oracle, rope_tables):
    """Small values in the first 256-token window, then values near the int32
    limit from token 300 on: the second window's magnitude sum does not fit,
    so it takes the reference's saturating recurrence after a summed first
    window."""
    rng = np.random.default_rng(13)
    ctx.kv_reset()
    pos = 420
    kv = oracle.kv_store(2, 4096)
    recs = {}
    for head in (6, 25):
        k8 = rng.integers(-5, 6, 128)
        recs[head] = [_record(k8, [2] * 4, rng.integers(-127, 128, 128), [24 if t >= 300 else 6] * 4)
                      for t in range(pos)]
    _write_records(ctx, kv, 0, recs)
    q, k, v = (_rand_q17(rng, 4096, 0.01) for _ in range(3))
    gq, ge = ctx.attention(0, pos, q, k, v)
    oq, oe = oracle.attention(kv, 2, 4096, 0, pos, oracle.rope(q, rope_tables, pos),
                              oracle.rope(k, rope_tables, pos), v)
    assert np.array_equal(gq, oq) and np.array_equal(ge, oe)
