"""Small, self-contained workloads for profiling single kernels (ncu).

  python -m 4pe_u250_b200.prof gemv --mode 4 --reps 3   one GEMV stage launch
  python -m 4pe_u250_b200.prof decode --layers 2         a few decode steps
  python -m 4pe_u250_b200.prof prefill --layers 32 --tokens 16
                                                         two prompt batches
  python -m 4pe_u250_b200.prof attention --context 4096 --reps 3
                                                         attention steps of one
                                                         layer over a filled cache
  python -m 4pe_u250_b200.prof sample --reps 3           device draws (top-p 0.9
                                                         and multinomial) over
                                                         32000 seeded logits
  python -m 4pe_u250_b200.prof pack --reps 1             one GATE projection and
                                                         the FP32 LM head packed
                                                         into bank images

Each builds a seeded synthetic model with only the layers it needs, so the
device footprint stays at a few hundred MB.
"""
import argparse
import importlib

import numpy as np


def kv_records(n, seed):
    """n synthetic KV records of one head: N(0, 1) K and V taken to Q15.17 and
    quantised by the reference's shift quantiser (the layout of
    swiftkv_attention.hpp:21-36), built in numpy."""
    rng = np.random.default_rng(seed)
    out = np.zeros((n, 320), np.uint8)
    for part, base in ((0, 64), (1, 192)):
        raw = np.clip(np.round(rng.standard_normal((n, 128)) * 131072.0), -2**31, 2**31 - 1).astype(np.int64)
        g = raw.reshape(n, 4, 32)
        mx = np.abs(g).max(axis=2)
        msb = np.floor(np.log2(np.maximum(mx, 1))).astype(np.int64)
        shift = np.where(mx == 0, 0, np.maximum(msb - 6, 0))
        mag = np.abs(g)
        half = np.where(shift > 0, 1 << np.maximum(shift - 1, 0), 0)[:, :, None]
        q = np.minimum((mag + half) >> shift[:, :, None], 127) * np.sign(g)
        out[:, base:base + 128] = q.reshape(n, 128).astype(np.int8).view(np.uint8)
        meta = np.zeros(n, np.uint64)
        for k in range(4):
            meta |= shift[:, k].astype(np.uint64) << np.uint64(5 * k + 20 * part)
        out[:, 0:8] |= meta.view(np.uint8).reshape(n, 8)
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("what", choices=["gemv", "decode", "prefill", "attention", "sample", "pack"])
    ap.add_argument("--mode", type=int, default=4)
    ap.add_argument("--layers", type=int, default=1)
    ap.add_argument("--reps", type=int, default=3)
    ap.add_argument("--tokens", type=int, default=4)
    ap.add_argument("--context", type=int, default=4096)
    a = ap.parse_args()
    pkg = importlib.import_module("4pe_u250_b200")
    synth = importlib.import_module("4pe_u250_b200.synth")
    F = pkg.formats
    if a.what == "attention":
        import torch
        with pkg.Context(num_layers=1, kv_capacity=a.context) as ctx:
            ctx.load_rope()
            for head in range(32):
                ctx.kv_write_tokens(head // 8, 0, head % 8, 0, kv_records(a.context - 1, 7 + head))
            rng = np.random.default_rng(3)
            qkv = torch.from_numpy(np.round(rng.standard_normal(3 * 4096) * 131072.0).astype(np.int32)).cuda()
            print(ctx.profile_attention(0, a.context - 1, qkv.data_ptr(), 0, a.reps))
        print("ok")
        return
    if a.what == "sample":
        import torch
        with pkg.Context(num_layers=1, kv_capacity=8) as ctx:
            logits = torch.from_numpy(np.random.default_rng(4).normal(0.0, 2.0, F.PADDED_VOCAB).astype(np.float32)).cuda()
            hist = np.random.default_rng(5).integers(0, F.VOCAB, 64).astype(np.int32)
            for top_p in (0.9, 0.0):
                smp = pkg.Sampler.make(0.8, top_p=top_p, repeat_penalty=1.1, seed=7)
                for _ in range(a.reps):
                    print(ctx.sample(logits.data_ptr(), hist, smp))
        print("ok")
        return
    if a.what == "pack":
        import torch
        with pkg.Context(num_layers=1, kv_capacity=8) as ctx:
            g = torch.Generator(device="cuda").manual_seed(6)
            imgs = [torch.zeros(F.BANK_BYTES, dtype=torch.uint8, device="cuda") for _ in range(4)]
            ptrs = [t.data_ptr() for t in imgs]
            rows, cols = 11008, 4096  # GATE, unpadded
            nib = torch.randint(0, 256, (rows * cols // 2,), dtype=torch.uint8, device="cuda", generator=g)
            sc = torch.rand(rows * cols // 128, device="cuda", generator=g) * 0.018 + 0.002
            head = torch.randn(32000 * 4096, device="cuda", generator=g) * 0.02
            for _ in range(a.reps):
                ctx.pack_autoround_matrix(0, F.MODE_GATE, nib.data_ptr(), sc.data_ptr(), ptrs)
                ctx.pack_fp32_head(head.data_ptr(), ptrs)
            torch.cuda.synchronize()
        print("ok")
        return
    banks = synth.model_banks(a.layers, 5)
    with pkg.Context(num_layers=a.layers, kv_capacity=64) as ctx:
        ctx.load_banks(banks)
        ctx.load_rope()
        if a.what == "gemv":
            x = synth.normal(F.mode_cols(a.mode), 0.0, 1.0, 5, synth.STREAM_INPUT)
            q, e = ctx.quantize_g32(x)
            for _ in range(a.reps):
                ctx.gemv(0, a.mode, q, e)
        elif a.what == "prefill":
            ctx.load_embeddings(synth.embeddings(5))
            ids = np.random.default_rng(1).integers(0, F.VOCAB, 2 * a.tokens).astype(np.int32)
            for b in range(2):
                print(ctx.prefill_tokens(b * a.tokens, ids[b * a.tokens:(b + 1) * a.tokens])[0])
        else:
            emb = synth.normal(a.tokens * 4096, 0.0, 0.02, 5, synth.STREAM_EMBEDDINGS)
            for pos in range(a.tokens):
                ctx.decode_token(pos, emb[pos * 4096:(pos + 1) * 4096])
    print("ok")


if __name__ == "__main__":
    main()
