"""Direct load of an AutoRound export onto the GPU.

Reads the AR4 stream that scripts/export_autoround_for_cpp.py writes
(``autoround_w4g128.bin``) and produces the four bank images on the device, as
scripts/autoround_pack_llama2_u250.py main() (:372-560) writes them to disk:
header (256 B: magic ``AR4\\0``, version, dim, hidden, layers, heads, KV heads,
vocabulary, group size), FP32 embeddings, then per layer the attention norm,
Q, K, V, O, the FFN norm, GATE, UP, DOWN (each projection: offset-binary
nibbles [rows][cols/2] then FP32 group-128 scales [rows][cols/128]), then the
final norm and the FP32 LM head.  Projections and the head are packed by
``i4d_pack_autoround_matrix`` / ``i4d_pack_fp32_head``; norm words are FP32
copies (bank p holds columns [1024p, 1024p+1024)).  The head takes the
script's max-abs RTN path (its calibrated ``--lm-head-autoround`` artifact is
not read here).  torch provides the device buffers.
"""
import struct

import numpy as np

from . import formats as F

HEADER_BYTES = 256
_PROJ = [(0, 4096, 4096), (1, 4096, 4096), (2, 4096, 4096), (3, 4096, 4096),
         (4, 11008, 4096), (5, 11008, 4096), (6, 4096, 11008)]


def read_header(f):
    h = f.read(HEADER_BYTES)
    if len(h) != HEADER_BYTES:
        raise ValueError("truncated AR4 header")
    magic, ver, dim, hidden, layers, heads, kv_heads, vocab, group = struct.unpack("<4sIIIIIIII", h[:36])
    if magic != b"AR4\0":
        raise ValueError(f"invalid magic {magic!r}")
    if (dim, hidden, vocab, group) != (4096, 11008, 32000, 128) or not 1 <= layers <= 32:
        raise ValueError(f"unsupported geometry dim={dim} hidden={hidden} vocab={vocab} group={group} layers={layers}")
    return {"version": ver, "dim": dim, "hidden": hidden, "layers": layers, "heads": heads,
            "kv_heads": kv_heads, "vocab": vocab, "group": group}


def _read(f, dtype, count):
    a = np.frombuffer(f.read(np.dtype(dtype).itemsize * count), dtype=dtype)
    if a.size != count:
        raise ValueError("truncated AR4 stream")
    return a


def _put_norm(images, layer, which, norm):
    import torch
    off = F.norm_word_offset(layer, which) * F.WORD_BYTES
    for p in range(4):
        part = torch.from_numpy(np.array(norm[p * 1024:(p + 1) * 1024]).view(np.uint8)).cuda()
        images[p][off:off + part.numel()] = part


def pack_autoround_file(ctx, path):
    """Returns (four device bank images as torch uint8 tensors, the FP32
    embeddings [32000][4096] as numpy, the header).  Layers beyond the
    header's count stay zero in the images."""
    import torch
    images = [torch.zeros(F.BANK_BYTES, dtype=torch.uint8, device="cuda") for _ in range(4)]
    ptrs = [t.data_ptr() for t in images]
    with open(path, "rb") as f:
        hdr = read_header(f)
        emb = _read(f, np.float32, 32000 * 4096).reshape(32000, 4096)
        for layer in range(hdr["layers"]):
            for mode, rows, cols in _PROJ:
                if mode == 0:
                    _put_norm(images, layer, 0, _read(f, np.float32, 4096))
                if mode == 4:
                    _put_norm(images, layer, 1, _read(f, np.float32, 4096))
                nib = torch.from_numpy(_read(f, np.uint8, rows * cols // 2).copy()).cuda()
                sc = torch.from_numpy(_read(f, np.float32, rows * cols // 128).copy()).cuda()
                ctx.pack_autoround_matrix(layer, mode, nib.data_ptr(), sc.data_ptr(), ptrs)
        _put_norm(images, 0, 2, _read(f, np.float32, 4096))
        head = torch.from_numpy(_read(f, np.float32, 32000 * 4096).copy()).cuda()
        ctx.pack_fp32_head(head.data_ptr(), ptrs)
    torch.cuda.synchronize()
    return images, emb, hdr
