"""CPU parity checkers (TEST INFRASTRUCTURE ONLY).

``Oracle`` wraps this repository's C restatement (oracle/i4d_oracle.c);
``RefEmulator`` wraps the unmodified reference emulator compiled from its own
source into oracle/_ref/ (present when the reference tree was available at
build time).  Only tests/, __graft_entry__.smoke() and bench.py's CPU
baseline use them; the product library never does.
"""
import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "_build", "libi4d_oracle.so")
REF_SO = os.path.join(HERE, "_ref", "libref_emulator.so")

P = ctypes.c_void_p


def _p(a):
    return None if a is None else a.ctypes.data


class Oracle:
    def __init__(self):
        if not os.path.exists(ORACLE_SO):
            raise RuntimeError(f"{ORACLE_SO} missing: run `make -C oracle`")
        L = ctypes.CDLL(ORACLE_SO)
        sigs = {
            "i4o_quantize_g32": [P, ctypes.c_int, P, P],
            "i4o_rmsnorm_quantize": [P, P, P, P, P],
            "i4o_linear_bank": [P, ctypes.c_int, ctypes.c_int, P, P, ctypes.c_int, P],
            "i4o_gemv": [P, ctypes.c_int, ctypes.c_int, P, P, P, P],
            "i4o_decode_rope_lut": [P, P, P],
            "i4o_rope_q17": [P, P, P],
            "i4o_kv_write_record": [P, P, P],
            "i4o_attention": [P, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, P, P, P, P, P],
            "i4o_swiglu": [P, P, ctypes.c_int, P],
            "i4o_read_gamma": [P, ctypes.c_int, ctypes.c_int, P],
            "i4o_forward": [P, P, P, P, ctypes.c_int, ctypes.c_int, ctypes.c_int, P, P],
            "i4o_float_to_q17_array": [P, ctypes.c_int, P],
            "i4o_expf_array": [P, P, ctypes.c_size_t],
            "i4o_argmax": [P, ctypes.c_int],
            "i4o_exp_negative_q17": [ctypes.c_int32],
            "i4o_sample": [ctypes.c_int, P, ctypes.c_int, P, ctypes.c_int, ctypes.c_float, ctypes.c_float,
                           ctypes.c_float, P],
            "i4o_nll": [P, ctypes.c_int, ctypes.c_int, P, P],
        }
        for k, v in sigs.items():
            getattr(L, k).argtypes = v
        L.i4o_argmax.restype = ctypes.c_int
        L.i4o_sample.restype = ctypes.c_int
        L.i4o_nll.restype = ctypes.c_double
        L.i4o_exp_negative_q17.restype = ctypes.c_uint32
        self.L = L
        self._rope = None

    @staticmethod
    def _banks(banks):
        return (ctypes.c_void_p * 4)(*[b.ctypes.data for b in banks])

    def quantize_g32(self, x):
        x = np.ascontiguousarray(x, dtype=np.float32)
        q = np.empty(x.size, np.int16)
        e = np.empty(x.size // 32, np.uint8)
        self.L.i4o_quantize_g32(x.ctypes.data, x.size, q.ctypes.data, e.ctypes.data)
        return q, e

    def rms_quant(self, x, gamma):
        x = np.ascontiguousarray(x, dtype=np.float32)
        g = np.ascontiguousarray(gamma, dtype=np.float32)
        q = np.empty(4096, np.int16)
        e = np.empty(128, np.uint8)
        r = np.empty(1, np.float32)
        self.L.i4o_rmsnorm_quantize(x.ctypes.data, g.ctypes.data, q.ctypes.data, e.ctypes.data, r.ctypes.data)
        return q, e, r[0]

    def linear_bank(self, superblocks, out_tiles, local_in_tiles, act_q, act_e, hls_zero_start=False):
        sb = np.ascontiguousarray(superblocks, dtype=np.uint8)
        q = np.ascontiguousarray(act_q, dtype=np.int16)
        e = np.ascontiguousarray(act_e, dtype=np.uint8)
        out = np.empty(out_tiles * 128, np.float32)
        self.L.i4o_linear_bank(sb.ctypes.data, out_tiles, local_in_tiles, q.ctypes.data, e.ctypes.data,
                               int(bool(hls_zero_start)), out.ctypes.data)
        return out

    def gemv(self, banks, layer, mode, act_q, act_e):
        from importlib import import_module
        F = import_module("4pe_u250_b200.formats")
        rows = F.mode_rows(mode)
        q = np.ascontiguousarray(act_q, dtype=np.int16)
        e = np.ascontiguousarray(act_e, dtype=np.uint8)
        y = np.empty(rows, np.float32)
        part = np.empty(4 * rows, np.float32)
        self.L.i4o_gemv(self._banks(banks), layer, mode, q.ctypes.data, e.ctypes.data, y.ctypes.data,
                        part.ctypes.data)
        return y, part.reshape(4, rows)

    def rope_tables(self, lut):
        buf = np.frombuffer(lut, dtype=np.uint8)
        c = np.empty(4096 * 64, np.int32)
        s = np.empty(4096 * 64, np.int32)
        self.L.i4o_decode_rope_lut(buf.ctypes.data, c.ctypes.data, s.ctypes.data)
        return c, s

    def float_to_q17(self, x):
        x = np.ascontiguousarray(x, dtype=np.float32)
        out = np.empty(x.size, np.int32)
        self.L.i4o_float_to_q17_array(x.ctypes.data, x.size, out.ctypes.data)
        return out

    def rope(self, vec, tables, pos):
        c, s = tables
        v = np.array(vec, dtype=np.int32, copy=True)
        self.L.i4o_rope_q17(v.ctypes.data, c[pos * 64:].ctypes.data, s[pos * 64:].ctypes.data)
        return v

    def kv_store(self, layers, stride):
        return np.zeros(4 * layers * 8 * stride * 320, np.uint8)

    def kv_record(self, k, v):
        rec = np.empty(320, np.uint8)
        k = np.ascontiguousarray(k, dtype=np.int32)
        v = np.ascontiguousarray(v, dtype=np.int32)
        self.L.i4o_kv_write_record(rec.ctypes.data, k.ctypes.data, v.ctypes.data)
        return rec

    def attention(self, kv, layers, stride, layer, pos, q_rot, k_rot, v):
        arrs = [np.ascontiguousarray(a, dtype=np.int32) for a in (q_rot, k_rot, v)]
        oq = np.empty(4096, np.int16)
        oe = np.empty(128, np.uint8)
        self.L.i4o_attention(kv.ctypes.data, layers, stride, layer, pos, *[a.ctypes.data for a in arrs],
                             oq.ctypes.data, oe.ctypes.data)
        return oq, oe

    def swiglu(self, gate, up):
        g = np.ascontiguousarray(gate, dtype=np.float32)
        u = np.ascontiguousarray(up, dtype=np.float32)
        out = np.empty(g.size, np.float32)
        self.L.i4o_swiglu(g.ctypes.data, u.ctypes.data, g.size, out.ctypes.data)
        return out

    def expf(self, x):
        x = np.ascontiguousarray(x, dtype=np.float32)
        y = np.empty_like(x)
        self.L.i4o_expf_array(x.ctypes.data, y.ctypes.data, x.size)
        return y

    def gamma(self, banks, layer, which):
        g = np.empty(4096, np.float32)
        self.L.i4o_read_gamma(self._banks(banks), layer, which, g.ctypes.data)
        return g

    def forward(self, banks, tables, kv, layers, stride, pos, residual):
        c, s = tables
        res = np.array(residual, dtype=np.float32, copy=True)
        logits = np.empty(32256, np.float32)
        self.L.i4o_forward(self._banks(banks), c.ctypes.data, s.ctypes.data, kv.ctypes.data, layers, stride, pos,
                           res.ctypes.data, logits.ctypes.data)
        return logits, res

    def argmax(self, logits, n=32000):
        x = np.ascontiguousarray(logits, dtype=np.float32)
        return self.L.i4o_argmax(x.ctypes.data, n)

    def nll(self, logits, target):
        """The perplexity loop's term for one position (emulator:1902-1926):
        (nll, max_l, sum_exp)."""
        x = np.ascontiguousarray(logits, dtype=np.float32)
        m, s = ctypes.c_float(0.0), ctypes.c_float(0.0)
        v = self.L.i4o_nll(x.ctypes.data, x.size, int(target), ctypes.byref(m), ctypes.byref(s))
        return v, m.value, s.value

    def sample(self, mode, logits, history, temperature, top_p, repeat_penalty, state):
        """One sampler draw (mode 0: decode_host.cpp:724-868, 1: emulator:1411-1569);
        returns (token, advanced state)."""
        x = np.ascontiguousarray(logits, dtype=np.float32)
        h = np.ascontiguousarray(history, dtype=np.int32)
        st = np.array([state], np.uint64)
        t = self.L.i4o_sample(mode, x.ctypes.data, x.size, h.ctypes.data if h.size else None, h.size,
                              temperature, top_p, repeat_penalty, st.ctypes.data)
        return t, int(st[0])


def pack_autoround_banks(mode, raw=None, scales=None, head=None):
    """CPU restatement of the reference packer for one matrix: the four banks'
    superblock bytes.  AutoRound matrices (modes 0-6): read_ar_matrix's unpack
    and Q1.15 scales (autoround_pack_llama2_u250.py:413-424), permute_qk_rows
    for Q/K (:101-113), zero padding (:483-488); the FP32 LM head (mode 7):
    pack_logits_into_banks' max-abs RTN (:268-307).  The superblock layout is
    the C restatement of pack_matrix_to_super_blocks in csrc/synth.c."""
    from importlib import import_module
    synth = import_module("4pe_u250_b200.synth")
    F = import_module("4pe_u250_b200.formats")
    rows = {0: 4096, 1: 4096, 2: 4096, 3: 4096, 4: 11264, 5: 11264, 6: 4096, 7: 32256}[mode]
    cols = 11264 if mode == 6 else 4096
    if mode == 7:
        M, K = head.shape
        hp = np.zeros((rows, cols), np.float32)
        hp[:M, :K] = head
        hr = hp.reshape(rows, cols // 128, 128)
        mx = np.maximum(np.max(np.abs(hr), axis=2, keepdims=True), np.float32(1e-8))
        sf = (mx / np.float32(7.0)).squeeze(axis=2)
        w = np.clip(np.round(hr / (sf[:, :, None] + np.float32(1e-12))), -8, 7).astype(np.int8).reshape(rows, cols)
        s = np.clip(np.round(sf * np.float32(32768.0)), -32768, 32767).astype(np.int16)
    else:
        M, K = raw.shape[0], raw.shape[1] * 2
        w0 = np.empty((M, K), np.int8)
        w0[:, 0::2] = (raw & 0x0F).astype(np.int8) - 8
        w0[:, 1::2] = (raw >> 4).astype(np.int8) - 8
        s0 = np.clip(np.round(scales * np.float32(32768.0)), -32768, 32767).astype(np.int16)
        if mode in (0, 1):
            perm = np.arange(4096).reshape(32, 128)
            src = np.empty_like(perm)
            src[:, 0::2] = perm[:, :64]
            src[:, 1::2] = perm[:, 64:]
            w0, s0 = w0[src.reshape(-1)], s0[src.reshape(-1)]
        w = np.zeros((rows, cols), np.int8)
        w[:M, :K] = w0
        s = np.zeros((rows, cols // 128), np.int16)
        s[:M, :K // 128] = s0
    return [synth.pack_arrays(w, s, p, rows // 128, cols // 1024) for p in range(4)]


def split_to_record(ks, vs, k8, v8):
    """Emulator split arrays (4 K shifts, 4 V shifts, K int8[128], V int8[128])
    -> the 320-byte record of swiftkv_attention.hpp:21-36."""
    rec = np.zeros(320, np.uint8)
    meta = 0
    for g in range(4):
        meta |= int(ks[g]) << (5 * g)
        meta |= int(vs[g]) << (20 + 5 * g)
    rec[0:8] = np.frombuffer(np.uint64(meta).tobytes(), np.uint8)
    rec[64:192] = np.asarray(k8, np.int8).view(np.uint8)
    rec[192:320] = np.asarray(v8, np.int8).view(np.uint8)
    return rec


def record_to_split(rec):
    rec = np.asarray(rec, np.uint8)
    meta = int(np.frombuffer(rec[0:8].tobytes(), np.uint64)[0])
    ks = np.array([(meta >> (5 * g)) & 31 for g in range(4)], np.uint8)
    vs = np.array([(meta >> (20 + 5 * g)) & 31 for g in range(4)], np.uint8)
    return ks, vs, rec[64:192].view(np.int8).copy(), rec[192:320].view(np.int8).copy()


def ref_available():
    return os.path.exists(REF_SO)


class RefEmulator:
    """The reference emulator itself (software_sim/llama2_decoder_sw_emulator.cpp).

    It holds one model and one KV state per process (its globals).
    """

    def __init__(self):
        if not ref_available():
            raise RuntimeError(f"{REF_SO} missing: build with `make -C oracle ref` where the reference exists")
        L = ctypes.CDLL(REF_SO)
        sigs = {
            "ref_load": [ctypes.c_char_p, ctypes.c_int, ctypes.c_int],
            "ref_kv_reset": [],
            "ref_threads": [],
            "ref_forward": [ctypes.c_int, ctypes.c_int, P, P],
            "ref_quantize_g32": [P, ctypes.c_int, P, P],
            "ref_rmsnorm_quantize": [P, P, P, P],
            "ref_gemv": [ctypes.c_int, ctypes.c_int, P, P, P],
            "ref_float_to_q17": [ctypes.c_float],
            "ref_rope_q17": [P, ctypes.c_int],
            "ref_attention": [P, P, P, ctypes.c_int, ctypes.c_int, P, P],
            "ref_swiglu": [P, P, ctypes.c_int, P],
            "ref_kv_get": [ctypes.c_int] * 4 + [P, P, P, P],
            "ref_kv_set": [ctypes.c_int] * 4 + [P, P, P, P],
            "ref_argmax": [P, ctypes.c_int],
            "ref_sample": [P, ctypes.c_int, P, ctypes.c_int, ctypes.c_float, ctypes.c_float, ctypes.c_float, P],
            "ref_perplexity": [ctypes.c_char_p, ctypes.c_int],
        }
        for k, v in sigs.items():
            getattr(L, k).argtypes = v
        L.ref_float_to_q17.restype = ctypes.c_int32
        self.L = L

    def sample(self, logits, history, temperature, top_p, repeat_penalty, state):
        """The emulator's own sampler (emulator:1411-1569): (token, advanced state)."""
        x = np.array(logits, dtype=np.float32)  # the emulator edits it
        h = np.ascontiguousarray(history, dtype=np.int32)
        st = (ctypes.c_ulonglong * 1)(state)
        t = self.L.ref_sample(x.ctypes.data, x.size, h.ctypes.data if h.size else None, h.size, temperature, top_p,
                              repeat_penalty, ctypes.addressof(st))
        return t, int(st[0])

    def perplexity(self, token_file, max_tokens=0):
        """The emulator's own calculate_perplexity (emulator:1775-1958) on an
        int32 token file ending in .bin; its report goes to stdout."""
        self.L.ref_perplexity(token_file.encode(), max_tokens)

    def load(self, directory, layers, stride):
        if self.L.ref_load(directory.encode(), layers, stride) != 0:
            raise RuntimeError(f"reference emulator could not load model from {directory}")

    def forward(self, token, pos):
        logits = np.empty(32000, np.float32)
        res = np.empty(4096, np.float32)
        self.L.ref_forward(token, pos, logits.ctypes.data, res.ctypes.data)
        return logits, res

    def gemv(self, layer, mode, q, e):
        from importlib import import_module
        F = import_module("4pe_u250_b200.formats")
        y = np.empty(F.mode_rows(mode), np.float32)
        q = np.ascontiguousarray(q, dtype=np.int16)
        e = np.ascontiguousarray(e, dtype=np.uint8)
        self.L.ref_gemv(layer, mode, q.ctypes.data, e.ctypes.data, y.ctypes.data)
        return y

    def rms_quant(self, x, gamma):
        x = np.ascontiguousarray(x, dtype=np.float32)
        g = np.ascontiguousarray(gamma, dtype=np.float32)
        q = np.empty(4096, np.int16)
        e = np.empty(128, np.uint8)
        self.L.ref_rmsnorm_quantize(x.ctypes.data, g.ctypes.data, q.ctypes.data, e.ctypes.data)
        return q, e

    def quantize_g32(self, x):
        x = np.ascontiguousarray(x, dtype=np.float32)
        q = np.empty(x.size, np.int16)
        e = np.empty(x.size // 32, np.uint8)
        self.L.ref_quantize_g32(x.ctypes.data, x.size, q.ctypes.data, e.ctypes.data)
        return q, e

    def attention(self, q_rot, k_rot, v, layer, pos):
        arrs = [np.ascontiguousarray(a, dtype=np.int32) for a in (q_rot, k_rot, v)]
        oq = np.empty(4096, np.int16)
        oe = np.empty(128, np.uint8)
        self.L.ref_attention(*[a.ctypes.data for a in arrs], layer, pos, oq.ctypes.data, oe.ctypes.data)
        return oq, oe

    def swiglu(self, gate, up):
        g = np.ascontiguousarray(gate, dtype=np.float32)
        u = np.ascontiguousarray(up, dtype=np.float32)
        out = np.empty(g.size, np.float32)
        self.L.ref_swiglu(g.ctypes.data, u.ctypes.data, g.size, out.ctypes.data)
        return out

    def kv_get(self, bank, layer, lh, token):
        k8 = np.empty(128, np.int8)
        v8 = np.empty(128, np.int8)
        ks = np.empty(4, np.uint8)
        vs = np.empty(4, np.uint8)
        self.L.ref_kv_get(bank, layer, lh, token, k8.ctypes.data, ks.ctypes.data, v8.ctypes.data, vs.ctypes.data)
        return ks, vs, k8, v8

    def kv_set(self, bank, layer, lh, token, ks, vs, k8, v8):
        """Writes one cached entry in the emulator's split arrays."""
        arrs = [np.ascontiguousarray(k8, np.int8), np.ascontiguousarray(ks, np.uint8),
                np.ascontiguousarray(v8, np.int8), np.ascontiguousarray(vs, np.uint8)]
        self.L.ref_kv_set(bank, layer, lh, token, *[a.ctypes.data for a in arrs])

    def kv_record(self, bank, layer, lh, token):
        """The cached entry as the 320-byte HLS record (metadata word: K shift
        of group g at bit 5g, V shift at 20 + 5g; K int8 at 64, V at 192)."""
        return split_to_record(*self.kv_get(bank, layer, lh, token))

    def kv_set_record(self, bank, layer, lh, token, rec):
        self.kv_set(bank, layer, lh, token, *record_to_split(rec))

    def argmax(self, logits):
        """The emulator's sample_argmax over 32000 logits (emulator:1428-1438)."""
        x = np.ascontiguousarray(logits, dtype=np.float32)
        return int(self.L.ref_argmax(x.ctypes.data, x.size))

    def threads(self):
        return self.L.ref_threads()
