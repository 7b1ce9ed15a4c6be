"""B200-native INT4 Llama-2-7B batch-1 decode (drop-in for the 4PE_U250 path).

Python/ctypes shim over ``libi4d.so`` (C ABI in include/i4d.h).  Mirrors the
reference host's operator surface: load the four bank images and the RoPE
LUT (decode_host.cpp:1236-1294), then one ``decode_token(position,
residual)`` per step returning the 32256 padded logits
(decode_host.cpp:1340-1556), plus the per-stage services used by parity
tests (linear stage, RMSNorm+quant, attention, SwiGLU+quant).

Errors raise I4DError carrying the C status and message; there is no CPU
fallback: without the CUDA library every call fails.
"""
import ctypes
import math
import os

import numpy as np

from . import formats

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libi4d.so")

OK, ERR_ARG, ERR_SIZE, ERR_CUDA, ERR_TIMEOUT, ERR_STATE, ERR_NOMEM = range(7)
FLAG_NO_GRAPH = 1
FLAG_NO_PDL = 2
FLAG_STAGED = 4

# Every symbol include/i4d.h declares.
EXPORTS = [
    "i4d_create", "i4d_destroy", "i4d_last_error", "i4d_load_bank", "i4d_load_rope",
    "i4d_load_embeddings", "i4d_decode_token", "i4d_kv_reset", "i4d_kv_read", "i4d_kv_write",
    "i4d_sync", "i4d_linear_bank", "i4d_gemv", "i4d_quantize_g32", "i4d_rms_quant",
    "i4d_attention", "i4d_swiglu_quant", "i4d_expf", "i4d_decode_token_async", "i4d_stream",
    "i4d_profile_token", "i4d_token_breakdown", "i4d_linear_bank_noalloc",
    "i4d_token_timeline", "i4d_create_shard", "i4d_shard_export", "i4d_shard_attach",
    "i4d_decode_greedy", "i4d_argmax", "i4d_sampler_init", "i4d_sample", "i4d_decode_sample",
    "i4d_pack_autoround_matrix", "i4d_pack_fp32_head", "i4d_prefill", "i4d_prefill_tokens", "i4d_eval_nll",
    "i4d_device_arch", "i4d_profile_gemv", "i4d_profile_attention", "i4d_kv_write_tokens",
]

SAMPLER_HOST = 0      # decode_host.cpp:724-868
SAMPLER_EMULATOR = 1  # emulator:1411-1569


class Sampler(ctypes.Structure):
    """i4d_sampler: temperature, top-p, repeat penalty, mode and the xorshift64*
    state that every coin flip advances (the reference Sampler's members)."""
    _fields_ = [("temperature", ctypes.c_float), ("top_p", ctypes.c_float), ("repeat_penalty", ctypes.c_float),
                ("mode", ctypes.c_int32), ("rng_state", ctypes.c_uint64)]

    @classmethod
    def make(cls, temperature, top_p=0.0, repeat_penalty=1.0, seed=0, mode=SAMPLER_HOST):
        s = cls()
        load_library().i4d_sampler_init(ctypes.byref(s), temperature, top_p, repeat_penalty, seed, mode)
        return s

_STAGES = ["qkv", "o", "gu", "down", "logits"]
BREAKDOWN = ([f"wait_{x}" for x in _STAGES] + [f"prologue_{x}" for x in _STAGES] + [f"chunks_{x}" for x in _STAGES]
             + ["attn_wait", "attn", "ring_full", "total"] + [f"arrive_{x}" for x in _STAGES]
             + [f"warp_{k}_{x}" for x in _STAGES for k in ("data_wait", "slot_wait", "compute", "chain")])

KERNEL_CLASSES = ["qkv_gemv", "attention", "o_gemv", "gate_up_gemv", "down_gemv", "logits_gemv", "rms", "token"]


def gather_handles(handle, group=None):
    """All ranks' shard handles in rank order, by a torch.distributed
    all-gather (any backend: the handles are host bytes)."""
    import torch.distributed as dist
    out = [None] * dist.get_world_size(group)
    dist.all_gather_object(out, handle, group=group)
    return out


class I4DError(RuntimeError):
    def __init__(self, status, message):
        super().__init__(f"i4d status {status}: {message}")
        self.status = status


class _Config(ctypes.Structure):
    _fields_ = [("device", ctypes.c_int), ("num_layers", ctypes.c_int),
                ("kv_capacity", ctypes.c_int), ("flags", ctypes.c_uint)]


_lib = None


def load_library():
    """Loads libi4d.so (raises if it was not built; no fallback exists)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise RuntimeError(f"{LIB_PATH} is missing: run __graft_entry__.build()")
    L = ctypes.CDLL(LIB_PATH)
    P = ctypes.c_void_p
    sig = {
        "i4d_create": [ctypes.POINTER(_Config), ctypes.POINTER(P)],
        "i4d_destroy": [P],
        "i4d_last_error": [P],
        "i4d_load_bank": [P, ctypes.c_int, P, ctypes.c_size_t],
        "i4d_load_rope": [P, P, ctypes.c_size_t],
        "i4d_load_embeddings": [P, P, ctypes.c_size_t],
        "i4d_decode_token": [P, ctypes.c_uint32, P, P, P],
        "i4d_kv_reset": [P],
        "i4d_kv_read": [P, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, P],
        "i4d_kv_write": [P, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, P],
        "i4d_sync": [P],
        "i4d_linear_bank": [P, P, ctypes.c_size_t, ctypes.c_int, ctypes.c_int, P, P, ctypes.c_int, P],
        "i4d_gemv": [P, ctypes.c_int, ctypes.c_int, P, P, P, P],
        "i4d_quantize_g32": [P, P, ctypes.c_int, P, P],
        "i4d_rms_quant": [P, P, P, P, P],
        "i4d_attention": [P, ctypes.c_int, ctypes.c_uint32, P, P, P, P, P],
        "i4d_swiglu_quant": [P, P, P, P, P],
        "i4d_expf": [P, P, P, ctypes.c_size_t],
        "i4d_device_arch": [ctypes.c_int, P, P],
        "i4d_kv_write_tokens": [P, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, P],
        "i4d_profile_gemv": [P, ctypes.c_int, ctypes.c_int, P],
        "i4d_profile_attention": [P, ctypes.c_int, ctypes.c_uint32, P, ctypes.c_int, ctypes.c_int, P],
        "i4d_decode_token_async": [P, ctypes.c_uint32, P, P],
        "i4d_stream": [P],
        "i4d_profile_token": [P, ctypes.c_uint32, P, P, P],
        "i4d_token_breakdown": [P, ctypes.c_uint32, P, P, ctypes.c_int],
        "i4d_linear_bank_noalloc": [P, P, ctypes.c_size_t, ctypes.c_int, ctypes.c_int, P, P, ctypes.c_int, P],
        "i4d_token_timeline": [P, ctypes.c_uint32, P, ctypes.c_int, ctypes.c_int, P, ctypes.c_int, P],
        "i4d_create_shard": [P, ctypes.c_int, ctypes.c_int, P],
        "i4d_shard_export": [P, P, ctypes.c_size_t],
        "i4d_shard_attach": [P, P, ctypes.c_size_t],
        "i4d_decode_greedy": [P, ctypes.c_uint32, ctypes.c_int32, P, P],
        "i4d_prefill": [P, ctypes.c_uint32, P, ctypes.c_uint32, P],
        "i4d_prefill_tokens": [P, ctypes.c_uint32, P, ctypes.c_uint32, P, P],
        "i4d_eval_nll": [P, P, ctypes.c_uint32, P],
        "i4d_argmax": [P, P, ctypes.c_size_t, P],
        "i4d_sample": [P, P, P, ctypes.c_uint32, P, P],
        "i4d_decode_sample": [P, ctypes.c_uint32, ctypes.c_int32, P, ctypes.c_uint32, P, P],
        "i4d_pack_autoround_matrix": [P, ctypes.c_int, ctypes.c_int, P, P, P],
        "i4d_pack_fp32_head": [P, P, P],
    }
    for name, args in sig.items():
        fn = getattr(L, name)
        fn.argtypes = args
        fn.restype = ctypes.c_int
    L.i4d_sampler_init.argtypes = [P, ctypes.c_float, ctypes.c_float, ctypes.c_float, ctypes.c_uint64, ctypes.c_int32]
    L.i4d_sampler_init.restype = None
    L.i4d_destroy.restype = None
    L.i4d_last_error.restype = ctypes.c_char_p
    L.i4d_stream.restype = ctypes.c_void_p
    _lib = L
    return L


def _ptr(a):
    return a.ctypes.data if a is not None else None


SHARD_HANDLE_BYTES = 64


def shard_banks(rank, world):
    """Banks held by `rank` of a bank-sharded group of `world` GPUs."""
    n = 4 // world
    return list(range(rank * n, rank * n + n))


def combine_bank_partials(partials):
    """The pair reducers and finalizer of the four bank partials of a GEMV
    (int4_linear_controller.cpp:1384-1439): y = (p0 + p1) + (p2 + p3) in
    FP32, the order the token kernel applies to the partials that a sharded
    group exchanges.  partials: [4][rows] float32, bank order."""
    p = np.asarray(partials, dtype=np.float32)
    return (p[0] + p[1]) + (p[2] + p[3])



def device_arch(device=0):
    """(binary architecture of the loaded token kernel, device compute
    capability), both as 10 * major + minor, queried through the C ABI."""
    L = load_library()
    b, cc = ctypes.c_int(0), ctypes.c_int(0)
    st = L.i4d_device_arch(device, ctypes.byref(b), ctypes.byref(cc))
    if st != OK:
        raise I4DError(st, "i4d_device_arch failed")
    return b.value, cc.value

class Context:
    """One decode context on one GPU (i4d_ctx).  With world > 1 it is rank
    `rank` of a bank-sharded group (i4d_create_shard): it holds the banks
    shard_banks(rank, world) and must be attached to its peers (attach_peers)
    before decoding."""

    def __init__(self, device=0, num_layers=32, kv_capacity=4096, flags=0, rank=0, world=1):
        self._L = load_library()
        cfg = _Config(device, num_layers, kv_capacity, flags)
        h = ctypes.c_void_p()
        if world == 1:
            st = self._L.i4d_create(ctypes.byref(cfg), ctypes.byref(h))
        else:
            st = self._L.i4d_create_shard(ctypes.byref(cfg), rank, world, ctypes.byref(h))
        if st != OK:
            raise I4DError(st, "i4d_create failed (see stderr)")
        self._h = h
        self.num_layers = num_layers
        self.kv_capacity = kv_capacity
        self.rank, self.world = rank, world
        self.banks = shard_banks(rank, world)

    # -- bank sharding ------------------------------------------------------
    def shard_handle(self):
        """This context's opaque peer handle (bytes)."""
        buf = ctypes.create_string_buffer(SHARD_HANDLE_BYTES)
        self._check(self._L.i4d_shard_export(self._h, buf, SHARD_HANDLE_BYTES))
        return buf.raw

    def attach_handles(self, handles):
        """Maps the peers from all ranks' handles, in rank order."""
        if len(handles) != self.world or any(len(x) != SHARD_HANDLE_BYTES for x in handles):
            raise I4DError(ERR_SIZE, "need one handle of SHARD_HANDLE_BYTES per rank")
        blob = b"".join(handles)
        self._check(self._L.i4d_shard_attach(self._h, blob, len(blob)))

    def attach_peers(self, group=None):
        """Exchanges handles over torch.distributed (all ranks call this)."""
        self.attach_handles(gather_handles(self.shard_handle(), group))

    def close(self):
        if getattr(self, "_h", None):
            self._L.i4d_destroy(self._h)
            self._h = None

    def __del__(self):
        self.close()

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def _check(self, st):
        if st != OK:
            raise I4DError(st, self._L.i4d_last_error(self._h).decode())

    # -- loading ----------------------------------------------------------
    def load_bank(self, bank, image):
        image = np.ascontiguousarray(image, dtype=np.uint8)
        self._check(self._L.i4d_load_bank(self._h, bank, image.ctypes.data, image.nbytes))

    def load_bank_device(self, bank, image_dev_ptr):
        """Load one bank image that is already in device memory (e.g. GPU-packed)."""
        self._check(self._L.i4d_load_bank(self._h, bank, image_dev_ptr, formats.BANK_BYTES))

    def pack_autoround_matrix(self, layer, mode, nibbles_dev_ptr, scales_dev_ptr, image_dev_ptrs):
        """Pack one AutoRound projection into four device bank images (i4d_pack_autoround_matrix)."""
        arr = (ctypes.c_void_p * 4)(*image_dev_ptrs)
        self._check(self._L.i4d_pack_autoround_matrix(self._h, layer, mode, nibbles_dev_ptr, scales_dev_ptr, arr))

    def pack_fp32_head(self, head_dev_ptr, image_dev_ptrs):
        """Quantise and pack an FP32 LM head into four device bank images (i4d_pack_fp32_head)."""
        arr = (ctypes.c_void_p * 4)(*image_dev_ptrs)
        self._check(self._L.i4d_pack_fp32_head(self._h, head_dev_ptr, arr))

    def load_banks(self, images):
        """Loads the held banks from the four images (the others are skipped)."""
        for p, img in enumerate(images):
            if p in self.banks:
                self.load_bank(p, img)

    def load_rope(self, lut=None):
        lut = formats.generate_rope_lut() if lut is None else lut
        buf = np.frombuffer(lut, dtype=np.uint8)
        self._check(self._L.i4d_load_rope(self._h, buf.ctypes.data, buf.nbytes))

    def load_embeddings(self, emb):
        emb = np.ascontiguousarray(emb, dtype=np.float32)
        self._check(self._L.i4d_load_embeddings(self._h, emb.ctypes.data, emb.size))

    # -- decode -----------------------------------------------------------
    def decode_token(self, position, residual_in, want_residual=False):
        x = np.ascontiguousarray(residual_in, dtype=np.float32)
        assert x.size == formats.DIM
        logits = np.empty(formats.PADDED_VOCAB, dtype=np.float32)
        res = np.empty(formats.DIM, dtype=np.float32) if want_residual else None
        self._check(self._L.i4d_decode_token(self._h, position, x.ctypes.data, logits.ctypes.data, _ptr(res)))
        return (logits, res) if want_residual else logits

    def decode_greedy(self, position, token_id, want_logits=False):
        """One greedy step from a token id (embeddings loaded): (next id, logits or None)."""
        nxt = ctypes.c_int32(0)
        logits = np.empty(formats.PADDED_VOCAB, dtype=np.float32) if want_logits else None
        self._check(self._L.i4d_decode_greedy(self._h, position, int(token_id), ctypes.byref(nxt), _ptr(logits)))
        return nxt.value, logits

    def prefill(self, position0, residuals_in):
        """A prompt from its embedding rows [n][4096] at positions position0..:
        the last token's 32256 padded logits; KV records of every token."""
        x = np.ascontiguousarray(residuals_in, dtype=np.float32).reshape(-1, formats.DIM)
        logits = np.empty(formats.PADDED_VOCAB, dtype=np.float32)
        self._check(self._L.i4d_prefill(self._h, position0, x.ctypes.data, x.shape[0], logits.ctypes.data))
        return logits

    def prefill_tokens(self, position0, token_ids, want_logits=False):
        """A prompt from token ids (embeddings loaded): (greedy next id, logits or None)."""
        ids = np.ascontiguousarray(token_ids, dtype=np.int32)
        nxt = ctypes.c_int32(0)
        logits = np.empty(formats.PADDED_VOCAB, dtype=np.float32) if want_logits else None
        self._check(self._L.i4d_prefill_tokens(self._h, position0, ids.ctypes.data, ids.size, ctypes.byref(nxt),
                                               _ptr(logits)))
        return nxt.value, logits

    def eval_nll(self, token_ids):
        """Per-position negative log-likelihoods of one chunk (n - 1 doubles)."""
        ids = np.ascontiguousarray(token_ids, dtype=np.int32)
        out = np.empty(max(ids.size - 1, 0), dtype=np.float64)
        self._check(self._L.i4d_eval_nll(self._h, ids.ctypes.data, ids.size, out.ctypes.data if out.size else None))
        return out

    def perplexity(self, token_ids, chunk=None):
        """The emulator's PPL loop (calculate_perplexity, emulator:1852-1944):
        chunks of `chunk` tokens (default: the KV capacity), each evaluated
        from position 0; returns (average loss, perplexity, tokens evaluated),
        the NLLs summed in order in double."""
        ids = np.ascontiguousarray(token_ids, dtype=np.int32)
        chunk = chunk or self.kv_capacity or 4096
        total, count = 0.0, 0
        for start in range(0, ids.size, chunk):
            part = ids[start:start + chunk]
            if part.size < 2:
                break
            for v in self.eval_nll(part):
                total += float(v)
                count += 1
        if count == 0:
            raise ValueError("needs at least 2 tokens")
        loss = total / count
        return loss, math.exp(loss), count

    def sample(self, logits_dev_ptr, history, sampler):
        """One device draw over 32000 logits at a device pointer; advances sampler.rng_state."""
        h = np.ascontiguousarray(history, dtype=np.int32)
        tok = ctypes.c_int32(0)
        self._check(self._L.i4d_sample(self._h, logits_dev_ptr, h.ctypes.data if h.size else None, h.size,
                                       ctypes.byref(sampler), ctypes.byref(tok)))
        return tok.value

    def decode_sample(self, position, token_id, history, sampler):
        """One decode step from a token id, then one device draw over its logits: the next id."""
        h = np.ascontiguousarray(history, dtype=np.int32)
        nxt = ctypes.c_int32(0)
        self._check(self._L.i4d_decode_sample(self._h, position, int(token_id), h.ctypes.data if h.size else None,
                                              h.size, ctypes.byref(sampler), ctypes.byref(nxt)))
        return nxt.value

    def argmax(self, logits):
        """The device argmax of i4d_decode_greedy over a host array."""
        x = np.ascontiguousarray(logits, dtype=np.float32)
        idx = ctypes.c_int32(0)
        self._check(self._L.i4d_argmax(self._h, x.ctypes.data, x.size, ctypes.byref(idx)))
        return idx.value

    def decode_token_async(self, position, residual_in_dev_ptr, logits_out_dev_ptr):
        """Enqueue one step on device pointers (e.g. torch tensor data_ptr())."""
        self._check(self._L.i4d_decode_token_async(self._h, position, residual_in_dev_ptr, logits_out_dev_ptr))

    def stream_handle(self):
        return self._L.i4d_stream(self._h)

    def profile_token(self, position, residual_in_dev_ptr):
        ms = np.zeros(8, np.float32)
        n = np.zeros(8, np.uint32)
        self._check(self._L.i4d_profile_token(self._h, position, residual_in_dev_ptr, ms.ctypes.data, n.ctypes.data))
        return {k: (float(ms[i]), int(n[i])) for i, k in enumerate(KERNEL_CLASSES)}

    def profile_gemv(self, mode, reps):
        """Milliseconds per GEMV of `mode`, `reps` launches over the layers' matrices in turn."""
        ms = ctypes.c_float(0.0)
        self._check(self._L.i4d_profile_gemv(self._h, mode, reps, ctypes.byref(ms)))
        return ms.value

    def profile_attention(self, layer, position, qkv_dev_ptr, fill, reps):
        """Milliseconds per attention step of `layer` at `position` (see i4d_profile_attention)."""
        ms = ctypes.c_float(0.0)
        self._check(self._L.i4d_profile_attention(self._h, layer, position, qkv_dev_ptr, fill, reps,
                                                  ctypes.byref(ms)))
        return ms.value

    def token_breakdown(self, position, residual_in_dev_ptr):
        """CTA-averaged microseconds per category of the persistent kernel."""
        out = np.zeros(len(BREAKDOWN), np.float32)
        self._check(self._L.i4d_token_breakdown(self._h, position, residual_in_dev_ptr, out.ctypes.data, out.size))
        return dict(zip(BREAKDOWN, out.tolist()))

    def token_timeline(self, position, residual_in_dev_ptr, layer, detail=False):
        """[CTAs, 162] global-timer stamps (ns) and counts of one layer (see i4d_token_timeline)."""
        out = np.zeros((1024, 218), np.uint64)
        n = ctypes.c_int(0)
        self._check(self._L.i4d_token_timeline(self._h, position, residual_in_dev_ptr, layer, int(bool(detail)),
                                               out.ctypes.data, out.shape[0], ctypes.byref(n)))
        return out[: n.value]

    def kv_reset(self):
        self._check(self._L.i4d_kv_reset(self._h))

    def kv_read(self, bank, layer, local_head, token):
        out = np.empty(formats.KV_RECORD_BYTES, dtype=np.uint8)
        self._check(self._L.i4d_kv_read(self._h, bank, layer, local_head, token, out.ctypes.data))
        return out

    def kv_write(self, bank, layer, local_head, token, record):
        rec = np.ascontiguousarray(record, dtype=np.uint8)
        assert rec.size == formats.KV_RECORD_BYTES
        self._check(self._L.i4d_kv_write(self._h, bank, layer, local_head, token, rec.ctypes.data))

    def kv_write_tokens(self, bank, layer, local_head, token0, records):
        """Records of tokens token0 .. token0 + n - 1 of one head ([n][320] bytes)."""
        rec = np.ascontiguousarray(records, dtype=np.uint8).reshape(-1, formats.KV_RECORD_BYTES)
        self._check(self._L.i4d_kv_write_tokens(self._h, bank, layer, local_head, token0, rec.shape[0],
                                                rec.ctypes.data))

    def sync(self):
        self._check(self._L.i4d_sync(self._h))

    # -- per-stage services -------------------------------------------------
    def linear_bank(self, superblocks, local_in_tiles, out_tiles, act_q, act_e8m0, hls_zero_start=False):
        sb = np.ascontiguousarray(superblocks, dtype=np.uint8)
        q = np.ascontiguousarray(act_q, dtype=np.int16)
        e = np.ascontiguousarray(act_e8m0, dtype=np.uint8)
        out = np.empty(out_tiles * 128, dtype=np.float32)
        self._check(self._L.i4d_linear_bank(self._h, sb.ctypes.data, sb.nbytes, local_in_tiles, out_tiles,
                                            q.ctypes.data, e.ctypes.data, int(bool(hls_zero_start)),
                                            out.ctypes.data))
        return out

    def linear_bank_noalloc(self, superblocks_dev_ptr, n_bytes, local_in_tiles, out_tiles, act_q_dev_ptr,
                            act_e8m0_dev_ptr, partial_out_dev_ptr, hls_zero_start=False):
        """i4d_linear_bank_noalloc on caller-owned device buffers (raw pointers)."""
        self._check(self._L.i4d_linear_bank_noalloc(self._h, superblocks_dev_ptr, n_bytes, local_in_tiles,
                                                    out_tiles, act_q_dev_ptr, act_e8m0_dev_ptr,
                                                    int(bool(hls_zero_start)), partial_out_dev_ptr))

    def gemv(self, layer, mode, act_q, act_e8m0, with_partials=False):
        rows = formats.mode_rows(mode)
        q = np.ascontiguousarray(act_q, dtype=np.int16)
        e = np.ascontiguousarray(act_e8m0, dtype=np.uint8)
        y = np.empty(rows, dtype=np.float32)
        part = np.empty(4 * rows, dtype=np.float32) if with_partials else None
        self._check(self._L.i4d_gemv(self._h, layer, mode, q.ctypes.data, e.ctypes.data, y.ctypes.data,
                                     _ptr(part)))
        return (y, part.reshape(4, rows)) if with_partials else y

    def quantize_g32(self, x):
        x = np.ascontiguousarray(x, dtype=np.float32)
        q = np.empty(x.size, dtype=np.int16)
        e = np.empty(x.size // 32, dtype=np.uint8)
        self._check(self._L.i4d_quantize_g32(self._h, x.ctypes.data, x.size, q.ctypes.data, e.ctypes.data))
        return q, e

    def rms_quant(self, x, gamma):
        x = np.ascontiguousarray(x, dtype=np.float32)
        g = np.ascontiguousarray(gamma, dtype=np.float32)
        q = np.empty(formats.DIM, dtype=np.int16)
        e = np.empty(formats.DIM // 32, dtype=np.uint8)
        self._check(self._L.i4d_rms_quant(self._h, x.ctypes.data, g.ctypes.data, q.ctypes.data, e.ctypes.data))
        return q, e

    def attention(self, layer, position, q, k, v):
        arrs = [np.ascontiguousarray(a, dtype=np.int32) for a in (q, k, v)]
        oq = np.empty(formats.DIM, dtype=np.int16)
        oe = np.empty(formats.DIM // 32, dtype=np.uint8)
        self._check(self._L.i4d_attention(self._h, layer, position, *[a.ctypes.data for a in arrs],
                                          oq.ctypes.data, oe.ctypes.data))
        return oq, oe

    def swiglu_quant(self, gate, up):
        g = np.ascontiguousarray(gate, dtype=np.float32)
        u = np.ascontiguousarray(up, dtype=np.float32)
        q = np.empty(formats.FFN, dtype=np.int16)
        e = np.empty(formats.FFN // 32, dtype=np.uint8)
        self._check(self._L.i4d_swiglu_quant(self._h, g.ctypes.data, u.ctypes.data, q.ctypes.data, e.ctypes.data))
        return q, e

    def expf(self, x):
        x = np.ascontiguousarray(x, dtype=np.float32)
        y = np.empty_like(x)
        self._check(self._L.i4d_expf(self._h, x.ctypes.data, y.ctypes.data, x.size))
        return y
