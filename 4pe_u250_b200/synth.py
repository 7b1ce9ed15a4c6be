"""Seeded synthetic model images (libi4d_synth.so) for tests and benchmarks.

The reference runs real AutoRound checkpoints that are absent here; every
workload uses random weights of the reference shapes and value ranges
(INT4 uniform in [-8, 7], Q1.15 scales from U[0.002, 0.02], gamma ~ N(1, 0.05),
embeddings ~ N(0, 0.02)) written in the exact bank format.
"""
import ctypes
import os

import numpy as np

from . import formats as F

_HERE = os.path.dirname(os.path.abspath(__file__))
_lib = None

# Random stream ids (any element of a stream is regenerated independently).
STREAM_EMBEDDINGS = 7000
STREAM_INPUT = 9000
STREAM_KV_K = 9100
STREAM_KV_V = 9200
STREAM_QKV = 9300


def lib():
    global _lib
    if _lib is None:
        path = os.path.join(_HERE, "libi4d_synth.so")
        if not os.path.exists(path):
            raise RuntimeError(f"{path} is missing: run __graft_entry__.build()")
        L = ctypes.CDLL(path)
        L.i4s_fill_model.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_uint64]
        L.i4s_fill_matrix.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_uint64]
        L.i4s_fill_norms.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_uint64]
        L.i4s_fill_normal.argtypes = [ctypes.c_void_p, ctypes.c_uint64, ctypes.c_float, ctypes.c_float,
                                      ctypes.c_uint64, ctypes.c_uint64]
        L.i4s_weight.argtypes = [ctypes.c_uint64, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int]
        L.i4s_scale.argtypes = [ctypes.c_uint64, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int]
        L.i4s_gamma.argtypes = [ctypes.c_void_p, ctypes.c_uint64, ctypes.c_int, ctypes.c_int]
        L.i4s_pack_arrays.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                      ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
        L.i4s_matrix_byte_offset.argtypes = [ctypes.c_int, ctypes.c_int]
        L.i4s_matrix_byte_offset.restype = ctypes.c_uint64
        _lib = L
    return _lib


def _ptrs(banks):
    return (ctypes.c_void_p * 4)(*[b.ctypes.data for b in banks])


def empty_banks():
    return [np.zeros(F.BANK_BYTES, dtype=np.uint8) for _ in range(4)]


def model_banks(layers, seed, banks=None):
    """Four bank images with layers [0, layers), the LM head and all norms."""
    banks = banks if banks is not None else empty_banks()
    lib().i4s_fill_model(_ptrs(banks), layers, seed)
    return banks


def fill_matrix(banks, layer, mode, seed):
    lib().i4s_fill_matrix(_ptrs(banks), layer, mode, seed)


def fill_norms(banks, layers, seed):
    lib().i4s_fill_norms(_ptrs(banks), layers, seed)


def normal(n, mean, std, seed, stream):
    out = np.empty(n, dtype=np.float32)
    lib().i4s_fill_normal(out.ctypes.data, n, mean, std, seed, stream)
    return out


def embeddings(seed):
    return normal(F.VOCAB * F.DIM, 0.0, 0.02, seed, STREAM_EMBEDDINGS)


def weight_matrix(seed, layer, mode, rows=None, cols=None):
    """Dense int8 weights of a synthetic matrix (slow path, small sizes only)."""
    rows = rows or F.mode_rows(mode)
    cols = cols or F.mode_cols(mode)
    L = lib()
    return np.array([[L.i4s_weight(seed, layer, mode, r, c) for c in range(cols)] for r in range(rows)],
                    dtype=np.int8)


def pack_arrays(w, s, bank, out_tiles, local_in_tiles):
    """C restatement of pack_matrix_to_super_blocks for dense arrays."""
    w = np.ascontiguousarray(w, dtype=np.int8)
    s = np.ascontiguousarray(s, dtype=np.int16)
    M, K = w.shape
    nbytes = out_tiles * local_in_tiles // 16 * F.SUPERBLOCK_WORDS * 64
    out = np.zeros(nbytes, dtype=np.uint8)
    lib().i4s_pack_arrays(w.ctypes.data, s.ctypes.data, M, K, bank, out_tiles, local_in_tiles, out.ctypes.data)
    return out
