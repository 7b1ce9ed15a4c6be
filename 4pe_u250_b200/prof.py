"""Small, self-contained workloads for profiling single kernels (ncu).

  python -m 4pe_u250_b200.prof gemv --mode 4 --reps 3   one GEMV stage launch
  python -m 4pe_u250_b200.prof decode --layers 2         a few decode steps
  python -m 4pe_u250_b200.prof prefill --layers 32 --tokens 16
                                                         two prompt batches

Each builds a seeded synthetic model with only the layers it needs, so the
device footprint stays at a few hundred MB.
"""
import argparse
import importlib

import numpy as np


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("what", choices=["gemv", "decode", "prefill"])
    ap.add_argument("--mode", type=int, default=4)
    ap.add_argument("--layers", type=int, default=1)
    ap.add_argument("--reps", type=int, default=3)
    ap.add_argument("--tokens", type=int, default=4)
    a = ap.parse_args()
    pkg = importlib.import_module("4pe_u250_b200")
    synth = importlib.import_module("4pe_u250_b200.synth")
    F = pkg.formats
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
